"""Graph builder, schedules, rewrites, profiling and the execution engine against the interpreter."""
import pytest
import torch

from brain_b200 import graph as G
from brain_b200 import graph_tools as T


def test_builders_schedule_and_summary():
    g = T.build_mlp_graph([8, 16, 16, 4], batch=3)
    x = torch.randn(3, 8)
    (y,) = T.run_graph(g, [x])
    assert y.shape == (3, 4)
    order = T.compute_topological_order(g)
    assert len(order) == len(g.nodes) and not T.analyze_cycles(g)
    s = T.generate_schedule(g)
    assert s.depth == len(g.nodes) and s.max_parallelism == 1  # a chain
    tg = T.build_transformer_graph(seq=5, dim=8, ffn=16)
    (out,) = T.run_graph(tg, [torch.randn(5, 8)])
    assert out.shape == (5, 8)
    par = T.analyze_parallelism(tg)
    assert par["max_parallelism"] >= 3  # the q, k, v projections are independent
    assert "linear" in T.format_graph_summary(tg) and sum(ln.startswith("  %") for ln in T.export_text(tg).splitlines()) == len(tg.nodes)
    assert T.total_output_memory_bytes(g) == 4 * 3 * (16 + 16 + 16 + 16 + 4)
    assert T.arithmetic_intensity(g) > 0
    assert isinstance(T.analyze_fusion_candidates(tg), list)


def test_rewrites_clone_profile_engine():
    b = T.GraphBuilder("rw")
    x = b.input("x", [4, 4])
    one = b.add_constant("one", torch.ones(4, 4))
    zero = b.add_constant("zero", torch.zeros(4, 4))
    h = b.op("mul", x, one)
    h = b.op("add", zero, h)
    h = b.op("identity", h)
    y = b.op("relu", h)
    z = b.op("exp", x)
    b.output(y, z)
    g = b.build()
    ref = T.run_graph(g, [torch.randn(4, 4, generator=torch.Generator().manual_seed(0))])
    assert T.rewrite_algebraic(g) == 3
    assert [n.op for n in g.nodes] == ["relu", "exp"]
    got = T.run_graph(g, [torch.randn(4, 4, generator=torch.Generator().manual_seed(0))])
    assert all(torch.equal(a, c) for a, c in zip(ref, got))
    sub = T.clone_subgraph(g, [g.outputs[1]])
    assert [n.op for n in sub.nodes] == ["exp"] and len(g.nodes) == 2
    prof = T.profile_graph(g, [torch.randn(4, 4)], iters=2)
    assert len(prof.per_node_ms) == 2 and prof.total_ms >= 0 and prof.top(1)[0][0] in ("relu", "exp")
    eng = T.ExecutionEngine(T.build_mlp_graph([8, 8], batch=2))
    xin = torch.randn(2, 8)
    assert torch.allclose(eng.run([xin])[0], T.run_graph(eng.g, [xin])[0])


@pytest.mark.gpu
def test_execution_engine_cuda_graph_replay():
    g = T.build_mlp_graph([64, 128, 32], batch=16)
    eng = T.ExecutionEngine(g)
    for seed in range(3):
        x = torch.randn(16, 64, device="cuda", generator=torch.Generator(device="cuda").manual_seed(seed))
        (y,) = eng.run([x])
        (ref,) = T.run_graph(g, [x])
        assert torch.allclose(y, ref, atol=1e-5)
    assert eng._graph is not None
