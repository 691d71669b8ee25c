"""Random number streams.

``manual_seed`` seeds PyTorch (CPU and CUDA generators) for every framework path. ``BrainRng``
reproduces the reference's xorshift128+ generator bit for bit (seeded through SplitMix64(seed+1),
``next_f64 = (u64 >> 11) * 2^-53``, ``randn`` = Box-Muller cosine branch;
crates/brain-core/src/random.rs:118-234 and crates/brain-core/src/tensor/impl.rs:222-236) so that
tests can regenerate exactly the tensors a reference run would use. The bulk generation runs in the
C++ runtime library (``csrc/codec.cpp``) with a pure-Python fallback.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from .. import _native

_native.register({"brain_rng_seed": ("brain_runtime", "lp"), "brain_rng_fill": ("brain_runtime", "plpi")})

_M64 = (1 << 64) - 1


def manual_seed(seed: int) -> None:
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    global _DEFAULT
    _DEFAULT = BrainRng.from_seed(seed)


class SplitMix64:
    def __init__(self, seed: int):
        self.state = seed & _M64

    def next_u64(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & _M64
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
        return z ^ (z >> 31)


class BrainRng:
    def __init__(self, s0: int, s1: int):
        if s0 == 0 and s1 == 0:
            s0, s1 = 0xDEADBEEFCAFEBABE, 0x123456789ABCDEF0
        self.state = [s0 & _M64, s1 & _M64]

    @staticmethod
    def from_seed(seed: int) -> "BrainRng":
        sm = SplitMix64((seed + 1) & _M64)
        return BrainRng(sm.next_u64(), sm.next_u64())

    def next_u64(self) -> int:
        s1, s0 = self.state
        result = (s0 + s1) & _M64
        self.state[0] = s0
        s1 = (s1 ^ (s1 << 23)) & _M64
        self.state[1] = s1 ^ s0 ^ (s1 >> 17) ^ (s0 >> 26)
        return result

    def next_u32(self) -> int:
        return self.next_u64() >> 32

    def next_f64(self) -> float:
        return (self.next_u64() >> 11) * (1.0 / 9007199254740992.0)

    def _fill(self, n: int, mode: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float64)
        if _native.available("brain_runtime"):
            st = (ctypes.c_uint64 * 2)(*self.state)
            f = _native.fn("brain_rng_fill")
            f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int]
            f(ctypes.addressof(st), n, out.ctypes.data, mode)
            self.state = [int(st[0]), int(st[1])]
            return out
        import math
        for i in range(n):
            if mode == 0:
                out[i] = self.next_f64()
            else:
                u1 = max(1.0 - self.next_f64(), 1e-15)
                u2 = self.next_f64()
                out[i] = math.sqrt(-2.0 * math.log(u1)) * math.cos(2.0 * math.pi * u2)
        return out

    def rand(self, *shape) -> torch.Tensor:
        n = int(np.prod(shape)) if shape else 1
        return torch.from_numpy(self._fill(n, 0)).reshape(shape)

    def randn(self, *shape) -> torch.Tensor:
        n = int(np.prod(shape)) if shape else 1
        return torch.from_numpy(self._fill(n, 1)).reshape(shape)


_DEFAULT = BrainRng.from_seed(0x123456789ABCDEF0)


def with_rng(fn):
    """Run fn(rng) with the thread's default reference-stream generator."""
    return fn(_DEFAULT)


LCG64_A = 6364136223846793005  # Knuth's MMIX multiplier and increment (public constants)
LCG64_C = 1442695040888963407


def lcg64_stream(state: int, count: int) -> np.ndarray:
    """The next ``count`` states of the 64-bit LCG s' = A s + C (mod 2^64) after ``state``, as uint64.
    Several reference crates draw from this generator one value at a time; here it is produced in
    blocks of 4096: within a block state_j = A_j s + C_j with (A_j, C_j) precomputed once, so each
    block is one vector multiply-add."""
    B = 4096
    a_j = np.empty(B, dtype=np.uint64)
    c_j = np.empty(B, dtype=np.uint64)
    a, c = 1, 0
    for j in range(B):
        a, c = (a * LCG64_A) & _M64, (c * LCG64_A + LCG64_C) & _M64
        a_j[j], c_j[j] = a, c
    out = np.empty(count, dtype=np.uint64)
    s = np.uint64(state & _M64)
    with np.errstate(over="ignore"):
        for b0 in range(0, count, B):
            blk = a_j * s + c_j
            k = min(B, count - b0)
            out[b0:b0 + k] = blk[:k]
            s = blk[B - 1]
    return out


def lcg64_unit(state: int, count: int) -> np.ndarray:
    """Uniform [0, 1) doubles (top 53 bits of each LCG state)."""
    return (lcg64_stream(state, count) >> np.uint64(11)).astype(np.float64) / float(1 << 53)
