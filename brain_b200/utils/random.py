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


# ------------------------------------------------------------------ further engines, seeding, distributions
# Reference: crates/brain-core/src/random.rs:55-100 (Rng trait: next_u64 = hi32 << 32 | lo32 for 32-bit
# engines, next_f32 = (u32 >> 8) 2^-24, fill_bytes little-endian u64 words), 145-190 (PCG32), 236-345
# (ChaCha8), 347-385 (SeedSeq), 387-640 (distributions), 642-700 (shuffle, global seed). The engines are
# the published algorithms: PCG32 is O'Neill's pcg32 (XSH-RR output, 64-bit LCG state, srandom-style
# seeding); ChaCha8 is Bernstein's ChaCha block function with 4 double rounds, a 64-bit block counter
# and a 64-bit nonce. Streams equal the reference's, so seeded host-side sampling reproduces its runs.

_M32 = (1 << 32) - 1


class Rng:
    """Shared output conversions over an engine's ``next_u32`` / ``next_u64``."""

    def next_u32(self) -> int:
        return self.next_u64() >> 32

    def next_u64(self) -> int:
        hi = self.next_u32()
        return (hi << 32) | self.next_u32()

    def next_f64(self) -> float:
        return (self.next_u64() >> 11) * (1.0 / 9007199254740992.0)

    def next_f32(self) -> float:
        return float(np.float32((self.next_u32() >> 8) * (1.0 / 16777216.0)))

    def fill_bytes(self, n: int) -> bytes:
        out = bytearray()
        while len(out) < n:
            out += self.next_u64().to_bytes(8, "little")
        return bytes(out[:n])

    def fill_f64(self, n: int) -> np.ndarray:
        return np.array([self.next_f64() for _ in range(n)], dtype=np.float64)


for _cls in (SplitMix64, BrainRng):  # the existing engines gain the shared conversions
    for _name in ("next_f32", "fill_bytes", "fill_f64"):
        setattr(_cls, _name, getattr(Rng, _name))
    if not hasattr(_cls, "next_f64"):
        _cls.next_f64 = Rng.next_f64
    if not hasattr(_cls, "next_u32"):
        _cls.next_u32 = Rng.next_u32
SplitMix64.split = lambda self: SplitMix64(self.next_u64())


class PCG32(Rng):
    MULT = 6364136223846793005
    DEFAULT_STREAM = 0x5446253602431CCB

    def __init__(self, seed: int, stream: int = DEFAULT_STREAM):
        self.state, self.inc = 0, ((stream << 1) | 1) & _M64
        self.next_u32()
        self.state = (self.state + seed) & _M64
        self.next_u32()

    @classmethod
    def from_seed(cls, seed: int) -> "PCG32":
        return cls(seed)

    def next_u32(self) -> int:
        old = self.state
        self.state = (old * self.MULT + self.inc) & _M64
        xs = (((old >> 18) ^ old) >> 27) & _M32
        rot = old >> 59
        return ((xs >> rot) | (xs << ((-rot) & 31))) & _M32


def _rotl32(v: int, n: int) -> int:
    return ((v << n) | (v >> (32 - n))) & _M32


class ChaCha8(Rng):
    _SIGMA = (0x61707865, 0x3320646E, 0x79622D32, 0x6B206574)  # "expand 32-byte k"

    def __init__(self, key: bytes, nonce: int):
        if len(key) != 32:
            raise ValueError("ChaCha8 key must be 32 bytes")
        words = [int.from_bytes(key[4 * i:4 * i + 4], "little") for i in range(8)]
        self.state = list(self._SIGMA) + words + [0, 0, nonce & _M32, (nonce >> 32) & _M32]
        self._refill()

    @classmethod
    def from_seed(cls, seed: int) -> "ChaCha8":
        sm = SplitMix64(seed)
        key = b"".join(sm.next_u64().to_bytes(8, "little") for _ in range(4))
        return cls(key, sm.next_u64())

    def _refill(self):
        x = list(self.state)

        def qr(a, b, c, d):
            x[a] = (x[a] + x[b]) & _M32
            x[d] = _rotl32(x[d] ^ x[a], 16)
            x[c] = (x[c] + x[d]) & _M32
            x[b] = _rotl32(x[b] ^ x[c], 12)
            x[a] = (x[a] + x[b]) & _M32
            x[d] = _rotl32(x[d] ^ x[a], 8)
            x[c] = (x[c] + x[d]) & _M32
            x[b] = _rotl32(x[b] ^ x[c], 7)
        for _ in range(4):
            for col in range(4):
                qr(col, 4 + col, 8 + col, 12 + col)
            for i in range(4):
                qr(i, 4 + (i + 1) % 4, 8 + (i + 2) % 4, 12 + (i + 3) % 4)
        self.buffer = [(x[i] + self.state[i]) & _M32 for i in range(16)]
        self.state[12] = (self.state[12] + 1) & _M32
        if self.state[12] == 0:
            self.state[13] = (self.state[13] + 1) & _M32
        self.index = 0

    def next_u32(self) -> int:
        if self.index >= 16:
            self._refill()
        v = self.buffer[self.index]
        self.index += 1
        return v


class SeedSeq:
    """Mixes a list of 32-bit entropy words into any number of 64-bit seeds (one SplitMix64 walk)."""

    def __init__(self, seeds):
        self.entropy = [int(s) & _M32 for s in seeds]

    @classmethod
    def from_u64(cls, seed: int) -> "SeedSeq":
        return cls([seed & _M32, (seed >> 32) & _M32])

    def generate_u64_seeds(self, count: int) -> list[int]:
        sm = SplitMix64(0x9E3779B97F4A7C15)
        for e in self.entropy:
            sm.state = (sm.state + e) & _M64
            sm.next_u64()
        return [sm.next_u64() for _ in range(count)]


class UniformDist:
    def __init__(self, low: float = 0.0, high: float = 1.0):
        if not low < high:
            raise ValueError("UniformDist: low must be < high")
        self.low, self.high = low, high

    @classmethod
    def standard(cls):
        return cls(0.0, 1.0)

    def sample(self, rng) -> float:
        return self.low + (self.high - self.low) * rng.next_f64()


class NormalDist:
    """Box-Muller (cosine branch, u1 = max(1 - U, 1e-15))."""

    def __init__(self, mean: float = 0.0, std: float = 1.0):
        if std < 0:
            raise ValueError("NormalDist: std must be non-negative")
        self.mean, self.std = mean, std

    @classmethod
    def standard(cls):
        return cls(0.0, 1.0)

    def sample(self, rng) -> float:
        import math
        if self.std == 0.0:
            return self.mean
        u1 = max(1.0 - rng.next_f64(), 1e-15)
        u2 = rng.next_f64()
        return self.mean + self.std * math.sqrt(-2.0 * math.log(u1)) * math.cos(2.0 * math.pi * u2)


class LogNormalDist:
    def __init__(self, mu: float, sigma: float):
        if sigma <= 0:
            raise ValueError("LogNormalDist: sigma must be > 0")
        self.mu, self.sigma = mu, sigma

    def sample(self, rng) -> float:
        import math
        return math.exp(NormalDist(self.mu, self.sigma).sample(rng))


class GammaDist:
    """Marsaglia-Tsang (2000) squeeze/rejection for shape >= 1; shape < 1 by the U^(1/shape) boost."""

    def __init__(self, shape: float, scale: float = 1.0):
        if shape <= 0 or scale <= 0:
            raise ValueError("GammaDist: shape and scale must be > 0")
        self.shape, self.scale = shape, scale

    def sample(self, rng) -> float:
        import math
        a = self.shape
        if a < 1.0:
            u = rng.next_f64()
            return GammaDist(a + 1.0, self.scale).sample(rng) * u ** (1.0 / a)
        d = a - 1.0 / 3.0
        c = 1.0 / math.sqrt(9.0 * d)
        n = NormalDist.standard()
        while True:
            z = n.sample(rng)
            v = (1.0 + c * z) ** 3
            if v <= 0.0:
                continue
            u = rng.next_f64()
            if u < 1.0 - 0.0331 * z ** 4 or math.log(u) < 0.5 * z * z + d * (1.0 - v + math.log(v)):
                return self.scale * d * v


class BetaDist:
    def __init__(self, alpha: float, beta: float):
        if alpha <= 0 or beta <= 0:
            raise ValueError("BetaDist parameters must be > 0")
        self.alpha, self.beta = alpha, beta

    def sample(self, rng) -> float:
        x = GammaDist(self.alpha).sample(rng)
        y = GammaDist(self.beta).sample(rng)
        return x / (x + y)


class ExponentialDist:
    def __init__(self, lam: float):
        if lam <= 0:
            raise ValueError("ExponentialDist: lambda must be > 0")
        self.lam = lam

    def sample(self, rng) -> float:
        import math
        return -math.log(max(1.0 - rng.next_f64(), 1e-15)) / self.lam


class CauchyDist:
    def __init__(self, location: float = 0.0, scale: float = 1.0):
        if scale <= 0:
            raise ValueError("CauchyDist: scale must be > 0")
        self.location, self.scale = location, scale

    def sample(self, rng) -> float:
        import math
        return self.location + self.scale * math.tan(math.pi * (rng.next_f64() - 0.5))


class BernoulliDist:
    def __init__(self, p: float):
        if not 0.0 <= p <= 1.0:
            raise ValueError("BernoulliDist: p must be in [0, 1]")
        self.p = p

    def sample_bool(self, rng) -> bool:
        return rng.next_f64() < self.p

    def sample(self, rng) -> float:
        return 1.0 if self.sample_bool(rng) else 0.0


class PoissonDist:
    """Knuth's multiplication method: count uniforms until their product drops to exp(-lambda)."""

    def __init__(self, lam: float):
        if lam <= 0:
            raise ValueError("PoissonDist: lambda must be > 0")
        self.lam = lam

    def sample(self, rng) -> int:
        import math
        limit, k, p = math.exp(-self.lam), 0, 1.0
        while True:
            k += 1
            p *= rng.next_f64()
            if p <= limit:
                return k - 1


class ShuffleSeq:
    """Fisher-Yates from the back, j = next_u64 mod (i + 1)."""

    @staticmethod
    def shuffle(seq: list, rng) -> list:
        for i in range(len(seq) - 1, 0, -1):
            j = rng.next_u64() % (i + 1)
            seq[i], seq[j] = seq[j], seq[i]
        return seq

    @staticmethod
    def randperm(n: int, rng) -> list[int]:
        return ShuffleSeq.shuffle(list(range(n)), rng)


_GLOBAL_SEED = 0x123456789ABCDEF0


def set_seed(seed: int) -> None:
    """Seed the default reference-stream generator and PyTorch's generators."""
    global _GLOBAL_SEED
    _GLOBAL_SEED = seed & _M64
    manual_seed(seed)


def get_seed() -> int:
    return _GLOBAL_SEED
