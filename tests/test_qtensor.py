"""QuantTensor / quantizers / per-token activation quantisation / magnitude pruning."""
import pytest
import torch

from brain_b200.quantization import QuantDType
from brain_b200.quantization import qtensor as Q


def test_scalar_helpers():
    s, z = Q.compute_scale_zero_point(-1.0, 3.0, 0, 255)
    assert s == pytest.approx(4 / 255) and z == round(1 / s)
    assert Q.dequantize_val(Q.quantize_val(1.0, s, z, 0, 255), s, z) == pytest.approx(1.0, abs=s)
    assert Q.compute_scale_zero_point(-2.0, 1.0, -127, 127, symmetric=True) == (2.0 / 127, 0)
    x = torch.arange(101.0)
    assert Q.minmax(x) == (0.0, 100.0) and Q.percentile_slice(x, 90) == pytest.approx(90.0)


@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("axis", [None, 0])
def test_quant_tensor_roundtrip(sym, axis):
    torch.manual_seed(0)
    x = torch.randn(8, 32) * torch.linspace(0.1, 3, 8)[:, None]
    qt = Q.QuantTensor.from_float(x, QuantDType.INT8 if sym else QuantDType.UINT8, sym, axis)
    back = qt.dequantize()
    scale = qt.qparams.scale if axis is None else qt.qparams.scale[:, None]
    assert ((back - x).abs() <= scale * 0.5 + 1e-6).all()
    assert qt.nbytes() == 256 and qt.shape == (8, 32)
    if sym:
        assert torch.equal(qt.qparams.zero_point, torch.zeros_like(qt.qparams.zero_point))


def test_act_quantizer_and_pruner():
    x = torch.tensor([[1.0, -2.0, 0.5], [100.0, 0.0, -50.0]])
    q, s = Q.quantize_per_token(x)
    assert q.dtype == torch.int8 and torch.allclose(s[:, 0], torch.tensor([2 / 127, 100 / 127]))
    assert q[0, 1] == -127 and q[1, 0] == 127
    aq = Q.ActQuantizer("per_tensor", momentum=0.5)
    aq.observe(torch.tensor([2.0]))
    aq.observe(torch.tensor([4.0]))
    assert aq.amax == 3.0
    q2, s2 = aq.quantize(torch.tensor([3.0, 6.0]))
    assert q2.tolist() == [127, 127] and float(s2) == pytest.approx(3 / 127)
    w = torch.arange(1.0, 11.0).reshape(2, 5)
    r = Q.MagnitudePruner(0.4).prune(w)
    assert r.sparsity == pytest.approx(0.4) and int((w == 0).sum()) == 4 and r.threshold == 4.0
    w2 = torch.tensor([[5.0, 1.0, 3.0, 2.0], [0.1, 0.4, 0.3, 0.2]])
    r2 = Q.MagnitudePruner(0.5, per_row=True).prune(w2)
    assert r2.mask.tolist() == [[True, False, True, False], [False, True, True, False]]
    with pytest.raises(ValueError):
        Q.MagnitudePruner(1.0)
    v = torch.tensor([-8, 7, 3, -1, 0], dtype=torch.int8)
    assert torch.equal(Q.unpack_i4_to_i8_buffer(Q.pack_i8_to_i4_buffer(v), 5), v)
    assert Q.f64_to_bf16(1.0 / 3).dtype == torch.bfloat16 and float(Q.bf16_to_f64(Q.f64_to_bf16(0.5))) == 0.5
    assert float(Q.f16_to_f64(Q.f64_to_f16(65504.0))) == 65504.0
