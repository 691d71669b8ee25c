"""Utilities: reference RNG streams, logging, profiling, configuration, safetensors, hashing."""
import zlib

from .config import ConfigManager, EnvConfig  # noqa: F401
from .logging import StandardLogger, get_logger  # noqa: F401
from .profiling import AtomicCounter, CudaTimer, Gauge, Profiler, ScopeGuard, TimingStats, max_over_ranks  # noqa: F401
from .random import BrainRng, SplitMix64, manual_seed, with_rng  # noqa: F401
from .safetensors import load_safetensors, save_safetensors  # noqa: F401


def fnv1a_64(data: bytes) -> int:
    h = 0xCBF29CE484222325
    for b in data:
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def adler32(data: bytes) -> int:
    return zlib.adler32(data) & 0xFFFFFFFF


def murmur3_32(data: bytes, seed: int = 0) -> int:
    """MurmurHash3 x86 32-bit (public-domain algorithm by Austin Appleby)."""
    c1, c2, m = 0xCC9E2D51, 0x1B873593, 0xFFFFFFFF
    h = seed & m
    n = len(data) // 4
    for i in range(n):
        k = int.from_bytes(data[4 * i:4 * i + 4], "little")
        k = (k * c1) & m
        k = ((k << 15) | (k >> 17)) & m
        k = (k * c2) & m
        h ^= k
        h = ((h << 13) | (h >> 19)) & m
        h = (h * 5 + 0xE6546B64) & m
    tail = data[4 * n:]
    k = 0
    for i, b in enumerate(tail):
        k |= b << (8 * i)
    if tail:
        k = (k * c1) & m
        k = ((k << 15) | (k >> 17)) & m
        k = (k * c2) & m
        h ^= k
    h ^= len(data)
    h ^= h >> 16
    h = (h * 0x85EBCA6B) & m
    h ^= h >> 13
    h = (h * 0xC2B2AE35) & m
    h ^= h >> 16
    return h
