"""Neuroevolution building blocks against restatements of crates/brain-neuroevolution/src
(benchmark.rs, crossover.rs, utils.rs, fitness.rs, ga/termination.rs, hyperneat/)."""
import math

import pytest
import torch

from brain_b200.zoo import neuro_extras as NX


def test_fast_rng_matches_xorshift64():
    r = NX.FastRng(0)
    x = 0x853C49E6748FEA9B
    M = (1 << 64) - 1
    for _ in range(5):
        x ^= (x << 13) & M
        x ^= x >> 7
        x ^= (x << 17) & M
        assert r.next_u64() == x
    g = NX.FastRng(42)
    v = g.sample_range(-1.0, 1.0)
    assert -1.0 <= v < 1.0


def test_benchmark_functions_batched():
    pop = torch.tensor([[0.0, 0.0], [1.0, 1.0], [1.0, 2.0]], dtype=torch.float64)
    assert NX.sphere_fn(pop).tolist() == [0.0, 2.0, 5.0]
    assert NX.rosenbrock_fn(pop).tolist() == [1.0, 0.0, 100.0]
    assert float(NX.rastrigin_fn(pop)[0]) == pytest.approx(0.0) and float(NX.ackley_fn(pop)[0]) == pytest.approx(0.0, abs=1e-12)
    x = [0.3, -1.2, 2.5]
    want = -20 * math.exp(-0.2 * math.sqrt(sum(v * v for v in x) / 3)) - math.exp(
        sum(math.cos(2 * math.pi * v) for v in x) / 3) + 20 + math.e
    assert float(NX.ackley_fn(torch.tensor([x], dtype=torch.float64))[0]) == pytest.approx(want)
    assert NX.rosenbrock_fn(torch.ones(2, 1)).tolist() == [0.0, 0.0]


def test_crossovers():
    a = torch.zeros(2, 5, dtype=torch.float64)
    b = torch.ones(2, 5, dtype=torch.float64)
    c1, c2 = NX.single_point_crossover(a, b, torch.tensor([2, 4]))
    assert c1[0].tolist() == [0, 0, 1, 1, 1] and c2[1].tolist() == [1, 1, 1, 1, 0]
    u = torch.tensor([[0.1, 0.9, 0.4, 0.6, 0.5]] * 2, dtype=torch.float64)
    c1, c2 = NX.uniform_crossover(a, b, u)
    assert c1[0].tolist() == [0, 1, 0, 1, 1] and torch.equal(c1 + c2, a + b)
    p1, p2 = torch.tensor([[1.0, 4.0]]), torch.tensor([[3.0, 2.0]])
    c1, c2 = NX.blx_alpha_crossover(p1, p2, 0.5, torch.zeros(1, 2), torch.ones(1, 2))
    assert c1.tolist() == [[0.0, 1.0]] and c2.tolist() == [[4.0, 5.0]]
    uu = torch.tensor([[0.25, 0.75]], dtype=torch.float64)
    c1, c2 = NX.sbx_crossover(p1.double(), p2.double(), 2.0, uu)
    for k, (x1, x2, uv) in enumerate(((1.0, 3.0, 0.25), (4.0, 2.0, 0.75))):
        beta = (2 * uv) ** (1 / 3) if uv <= 0.5 else (1 / (2 * (1 - uv))) ** (1 / 3)
        assert float(c1[0, k]) == pytest.approx(0.5 * ((1 + beta) * x1 + (1 - beta) * x2))
        assert float(c2[0, k]) == pytest.approx(0.5 * ((1 - beta) * x1 + (1 + beta) * x2))
    assert torch.allclose(c1 + c2, p1.double() + p2.double())  # SBX preserves the parents' mean


def test_ranking_stats_termination_and_parallel_eval():
    assert NX.rank_fitness([0.5, 2.0, 2.0, -1.0]) == [1, 2, 0, 3]
    st = NX.FitnessStats.from_fitnesses([3.0, 1.0, 2.0, 10.0])
    assert (st.best, st.worst, st.median, st.mean) == (10.0, 1.0, 2.5, 4.0)
    cfg = NX.TerminationConfig(patience=2, target_fitness=5.0)
    tr = NX.TerminationTracker()
    assert not tr.update(1.0, cfg) and not tr.update(1.00001, cfg) and tr.update(1.0, cfg)
    assert NX.TerminationTracker().update(6.0, cfg)
    pop = torch.randn(100, 4)
    torch.testing.assert_close(NX.evaluate_population_parallel(pop, NX.sphere_fn, chunk=32), NX.sphere_fn(pop))


def test_cppn_substrate_and_checkpoint(tmp_path):
    sub = NX.SubstrateGrid2D(3, 2, 2, 1)
    assert sub.in_coords.tolist()[:3] == [[-1.0, -1.0], [0.0, -1.0], [1.0, -1.0]] and sub.out_coords.tolist() == [[-1.0, 0.0], [1.0, 0.0]]
    w = sub.generate_weight_matrix(NX.Cppn())
    assert w.shape == (2, 6)
    x1, y1 = sub.in_coords[4].tolist()
    x2, y2 = sub.out_coords[1].tolist()
    assert float(w[1, 4]) == pytest.approx(math.exp(-((x2 - x1) ** 2 + (y2 - y1) ** 2)) - 0.5)
    torch.testing.assert_close(sub.generate_weight_matrix(NX.Cppn.default()), w)
    m = NX.Cppn.default().mutate(torch.Generator().manual_seed(0))
    assert not torch.allclose(sub.generate_weight_matrix(m), w)
    thr = sub.generate_weight_matrix(NX.Cppn(), threshold=0.3)
    assert bool(((thr == 0) | (thr.abs() > 0.3)).all())
    ck = NX.EvoCheckpoint(3, torch.randn(4, 2), torch.randn(4), torch.randn(2), 1.5)
    p = str(tmp_path / "evo.pt")
    ck.save(p)
    back = NX.EvoCheckpoint.load(p)
    assert back.generation == 3 and torch.equal(back.population, ck.population) and back.best_fitness == 1.5
