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


def test_onnx_entry_points(tmp_path):
    from brain_b200 import onnx as O
    data = O.create_mlp_zoo_model((4, 8, 2))
    summ = O.onnx_summary(data)
    assert summ["nodes"] == 3 and summ["parameters"] == 4 * 8 + 8 + 8 * 2 + 2 and summ["problems"] == []
    x = torch.randn(1, 4)
    ref = T.run_graph(T.build_mlp_graph([4, 8, 2]), [x])[0]
    assert torch.allclose(O.evaluate_onnx_model(data, [x])[0], ref, atol=1e-6)
    p = tmp_path / "m.onnx"
    p.write_bytes(data)
    assert len(O.load_onnx(str(p)).nodes) == 3
    # matmul + bias add -> one linear
    b = T.GraphBuilder("mm")
    xi = b.input("x", [2, 3])
    w = b.add_constant("w", torch.randn(3, 5))
    bias = b.add_constant("b", torch.randn(5))
    y = b.op("relu", b.op("add", b.op("matmul", xi, w), bias))
    b.output(y)
    g = b.build()
    xin = torch.randn(2, 3)
    before = T.run_graph(g, [xin])[0]
    assert O.fuse_matmul_add(g) == 1 and [n.op for n in g.nodes] == ["linear", "relu"]
    assert torch.allclose(T.run_graph(g, [xin])[0], before, atol=1e-6)
    assert len(O.import_and_optimize(O.lower_from_graph_ir(g)).nodes) == 2
    v = 300
    enc = O.encode_varint(v)
    assert O.decode_varint(enc) == (300, 2) and O.default_opset() == 17 and O.is_valid_opset(13)
    assert O.read_f32_le(struct_pack_f(1.5)) == 1.5 and O.compute_crc32(b"123456789") == 0xCBF43926


def struct_pack_f(x):
    import struct
    return struct.pack("<f", x)


def test_exporters_and_builder(tmp_path):
    from brain_b200 import export as E
    g = T.build_mlp_graph([4, 8, 2])
    for fmt in ("onnx", "webnn", "tflite", "coreml"):
        p = E.export_model(g, fmt, str(tmp_path / f"m.{fmt}"))
        assert (tmp_path / f"m.{fmt}").stat().st_size > 0 and p.endswith(fmt)
    assert E.is_op_supported("linear", E.ExportFormat.ONNX)
    assert E.map_dtype_to_onnx(torch.bfloat16) == 16 and E.map_dtype_to_tflite(torch.int8) == 9
    assert E.sanitize_name("1 layer.w") == "_1_layer_w" and E.align4(5) == 8
    assert E.encode_uleb128(624485) == bytes([0xE5, 0x8E, 0x26])
    ar = E.SafetensorsArchive().add("w", torch.arange(4.0))
    ar.metadata["step"] = 3
    ar.save(str(tmp_path / "a.safetensors"))
    back = E.SafetensorsArchive.load(str(tmp_path / "a.safetensors"))
    assert torch.equal(back.tensors["w"], torch.arange(4.0)) and back.metadata.get("step") == "3"
