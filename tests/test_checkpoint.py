"""Checkpoint formats: byte layouts, CRC32 tamper detection and bit-exact round trips.

Mirrors the reference's checkpoint tests (crates/brain-train/tests/trainer_regression.rs:99-190,
crates/brain-export/tests/export_test.rs): save -> load -> save is byte-identical, values are
bit-exact, and a flipped byte is rejected.
"""
import math
import struct

import numpy as np
import pytest
import torch

from brain_b200.checkpoint import formats as F


def test_crc32_known_vector():
    assert F.crc32(b"123456789") == 0xCBF43926
    assert F.crc32(b"") == 0
    # streaming == one shot
    s = F.crc32(b"1234", state=0xFFFFFFFF)
    s = F.crc32(b"56789", state=s)
    assert s ^ 0xFFFFFFFF == 0xCBF43926


@pytest.mark.parametrize("v,expected", [
    (0.1, "0.1"), (1.0, "1"), (-2.5, "-2.5"), (1e-7, "0.0000001"), (1e21, "1000000000000000000000"),
    (-0.0, "-0"), (0.0, "0"), (float("nan"), "NaN"), (float("inf"), "inf"), (float("-inf"), "-inf"),
    (0.1 + 0.2, "0.30000000000000004"), (123456.789, "123456.789"), (3.0e-5, "0.00003"),
    (1.5e300, "15" + "0" * 299),
])
def test_rust_display_format(v, expected):
    assert F.format_f64(np.array([v])) == expected
    assert F._rust_display(v) == expected  # pure-python fallback agrees


def test_format_parse_roundtrip_bit_exact():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(2000) * 10.0 ** rng.integers(-30, 30, 2000),
                           [5e-324, 1.7976931348623157e308, -1e-310, 0.0, -0.0]])
    txt = F.format_f64(vals)
    assert "e" not in txt
    back = F.parse_f64(txt)
    assert back.tobytes() == vals.tobytes()
    with pytest.raises(F.CheckpointError):
        F.parse_f64("1.0,abc")


def test_tensor_v2_layout_and_tamper():
    t = torch.arange(6, dtype=torch.float32).reshape(2, 3)
    b = F.serialize_tensor(t)
    assert b[:8] == b"BRAIN   "
    assert struct.unpack_from("<I", b, 8)[0] == 2
    assert b[12] == 0 and b[13] == F.DTYPE_CODES["f32"]
    assert struct.unpack_from("<I", b, 16)[0] == 2
    assert struct.unpack_from("<2Q", b, 20) == (2, 3)
    plen = struct.unpack_from("<Q", b, 40)[0]
    assert plen == 48 and len(b) == 48 + 48
    back, tag = F.deserialize_tensor(b, return_tag=True)
    assert tag == "f32" and torch.equal(back, t.double())
    bad = bytearray(b)
    bad[-1] ^= 0x40
    with pytest.raises(F.CheckpointError, match="CRC32"):
        F.deserialize_tensor(bytes(bad))


def test_tensor_v1_read():
    data = np.array([1.5, -2.0], dtype="<f8")
    b = b"BRAIN   " + struct.pack("<I", 1) + bytes([1]) + struct.pack("<I", 1) + struct.pack("<Q", 2) + data.tobytes()
    t = F.deserialize_tensor(b)
    assert t.tolist() == [1.5, -2.0]


def test_archive_and_bn_roundtrip_and_tamper():
    a = F.TensorArchive()
    a.add("w", torch.randn(3, 4, dtype=torch.float64))
    a.add("b", torch.zeros(4, dtype=torch.float64))
    b1 = a.serialize()
    a2 = F.TensorArchive.deserialize(b1)
    assert a2.serialize() == b1
    m = F.BrainModelFile("net").with_meta("arch", "mlp")
    m.add_tensor("layer.0", torch.ones(2, 2, dtype=torch.float64), F.NodeCoord3D(1, 2, 3))
    bb = m.to_bytes()
    m2 = F.BrainModelFile.from_bytes(bb)
    assert m2.name == "net" and m2.metadata == {"arch": "mlp"} and m2.node_coords["layer.0"] == F.NodeCoord3D(1, 2, 3)
    assert m2.to_bytes() == bb
    bad = bytearray(bb)
    bad[20] ^= 1
    with pytest.raises(F.CheckpointError):
        F.BrainModelFile.from_bytes(bytes(bad))


def test_model_state_text_roundtrip_bit_exact(tmp_path):
    torch.manual_seed(0)
    lin = torch.nn.Sequential(torch.nn.Linear(5, 7), torch.nn.Linear(7, 2))
    st = F.ModelState.from_module(lin, {"optimizer_steps": 3, "format": "brain-train-state-v1"})
    p = tmp_path / "m.brain"
    st.save_file(str(p))
    raw = p.read_bytes()
    assert raw.startswith(b"BRAIN_STATE_V1\nmeta|format|brain-train-state-v1\nmeta|optimizer_steps|3\ntensor|0.weight|7x5|")
    st2 = F.ModelState.load_file(str(p))
    assert st2.to_brain_bytes() == raw
    for a, b in zip(st.tensors, st2.tensors):
        assert a.name == b.name
        assert torch.equal(a.tensor.double(), b.tensor)
    lin2 = torch.nn.Sequential(torch.nn.Linear(5, 7), torch.nn.Linear(7, 2))
    st2.load_into(lin2)
    for x, y in zip(lin.parameters(), lin2.parameters()):
        assert torch.equal(x, y)
    # bf16 values survive exactly through the f64 text
    bt = torch.randn(64).bfloat16()
    s3 = F.ModelState([F.NamedTensor("x", bt)], {})
    back = F.ModelState.from_brain_bytes(s3.to_brain_bytes()).tensors[0].tensor
    assert torch.equal(back.bfloat16(), bt)
    with pytest.raises(F.CheckpointError):
        F.ModelState.from_brain_bytes(b"NOT_A_STATE\n")
    with pytest.raises(F.CheckpointError):
        F.ModelState.from_brain_bytes(b"BRAIN_STATE_V1\ntensor|x|2|1.0,zz\n")
    with pytest.raises(F.CheckpointError):
        F.ModelState.from_brain_bytes(b"BRAIN_STATE_V1\ntensor|x|2a|1.0\n")


def test_scalar_tensor_shape_empty():
    st = F.ModelState([F.NamedTensor("s", torch.tensor(2.5, dtype=torch.float64))], {})
    b = st.to_brain_bytes()
    assert b"tensor|s||2.5" in b
    assert F.ModelState.from_brain_bytes(b).tensors[0].tensor.shape == ()


def test_brain_v2_native_dtypes(tmp_path):
    ts = {"a": torch.randn(33, 7).bfloat16(), "b": torch.randn(5), "c": torch.arange(10, dtype=torch.int64),
          "d": torch.randn(16).to(torch.float8_e4m3fn)}
    p = str(tmp_path / "ck.brain")
    F.save_brain_v2(p, ts, {"step": 7})
    raw1 = open(p, "rb").read()
    back, meta = F.load_brain_v2(p)
    assert meta == {"step": 7}
    for k in ts:
        assert back[k].dtype == ts[k].dtype
        assert torch.equal(back[k].view(torch.uint8), ts[k].view(torch.uint8))
    F.save_brain_v2(p, back, meta)
    assert open(p, "rb").read() == raw1
    bad = bytearray(raw1)
    bad[-3] ^= 0xFF
    open(p, "wb").write(bytes(bad))
    with pytest.raises(F.CheckpointError):
        F.load_brain_v2(p)
