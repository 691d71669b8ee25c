"""Reference PRNG engines against their published test vectors, and the distributions' moments."""
import math

import pytest

from brain_b200.utils import random as r


def test_pcg32_published_vector():
    # pcg32 demo (seed 42, stream 54): the first outputs of O'Neill's reference implementation
    p = r.PCG32(42, 54)
    assert [p.next_u32() for _ in range(6)] == [0xa15c02b7, 0x7b47f409, 0xba1d3330, 0x83d2f293, 0xbfa4784b,
                                                0xcbed606e]
    a, b = r.PCG32.from_seed(7), r.PCG32.from_seed(7)
    assert [a.next_u64() for _ in range(4)] == [b.next_u64() for _ in range(4)]


def test_chacha8_published_keystream():
    # ChaCha8, all-zero key and nonce: keystream bytes 3e 00 ef 2f 89 5f 40 d6 7f 5b b8 e8 1f 09 a5 a1
    c = r.ChaCha8(bytes(32), 0)
    got = b"".join(c.next_u32().to_bytes(4, "little") for _ in range(4))
    assert got.hex() == "3e00ef2f895f40d67f5bb8e81f09a5a1"
    c2 = r.ChaCha8(bytes(32), 0)
    words = [c2.next_u32() for _ in range(40)]  # crosses two block refills
    assert len(set(words)) == 40
    with pytest.raises(ValueError):
        r.ChaCha8(bytes(16), 0)


def test_seed_seq_and_engine_conversions():
    s = r.SeedSeq.from_u64(0x1234_5678_9abc_def0)
    assert s.entropy == [0x9abcdef0, 0x12345678]
    a = s.generate_u64_seeds(4)
    assert a == r.SeedSeq([0x9abcdef0, 0x12345678]).generate_u64_seeds(4) and len(set(a)) == 4
    assert a != r.SeedSeq([1, 2]).generate_u64_seeds(4)
    sm = r.SplitMix64(3)
    child = sm.split()
    assert isinstance(child, r.SplitMix64) and child.next_u64() != sm.next_u64()
    g = r.BrainRng.from_seed(5)
    assert len(g.fill_bytes(13)) == 13 and 0.0 <= g.next_f32() < 1.0


@pytest.mark.parametrize("dist,mean,var", [
    (r.UniformDist(2.0, 4.0), 3.0, 4.0 / 12),
    (r.NormalDist(1.0, 2.0), 1.0, 4.0),
    (r.LogNormalDist(0.0, 0.5), math.exp(0.125), (math.exp(0.25) - 1) * math.exp(0.25)),
    (r.GammaDist(3.0, 2.0), 6.0, 12.0),
    (r.GammaDist(0.5, 1.0), 0.5, 0.5),
    (r.BetaDist(2.0, 5.0), 2 / 7, 10 / (49 * 8)),
    (r.ExponentialDist(4.0), 0.25, 1 / 16),
    (r.BernoulliDist(0.3), 0.3, 0.21),
    (r.PoissonDist(3.5), 3.5, 3.5),
])
def test_distribution_moments(dist, mean, var):
    rng = r.PCG32.from_seed(11)
    n = 40000
    xs = [float(dist.sample(rng)) for _ in range(n)]
    m = sum(xs) / n
    v = sum((x - m) ** 2 for x in xs) / (n - 1)
    assert abs(m - mean) < 5 * math.sqrt(var / n)
    assert abs(v - var) < 0.06 * var


def test_cauchy_median_and_shuffle():
    rng = r.ChaCha8.from_seed(2)
    xs = sorted(r.CauchyDist(1.0, 0.5).sample(rng) for _ in range(20001))
    assert abs(xs[10000] - 1.0) < 0.05
    q1, q3 = xs[5000], xs[15000]
    assert abs((q3 - q1) - 1.0) < 0.06  # interquartile range = 2 scale
    perm = r.ShuffleSeq.randperm(50, r.BrainRng.from_seed(1))
    assert sorted(perm) == list(range(50)) and perm != list(range(50))
    assert r.ShuffleSeq.randperm(50, r.BrainRng.from_seed(1)) == perm
    r.set_seed(99)
    assert r.get_seed() == 99
    for bad in (lambda: r.UniformDist(1, 1), lambda: r.GammaDist(0), lambda: r.BernoulliDist(1.5),
                lambda: r.PoissonDist(0), lambda: r.NormalDist(0, -1)):
        with pytest.raises(ValueError):
            bad()
