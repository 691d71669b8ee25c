"""FP8 block-scaled GEMM (tcgen05 kind::f8f6f4 with software promotion) and quantisation."""
import pytest
import torch

from brain_b200 import quantization as Q
from brain_b200.quantization import fp8 as F8


def _rnd(*s, seed=0, scale=1.0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*s, generator=g) * scale).to(device)


def test_fp8_roundtrip_cpu():
    x = _rnd(64, 256, seed=1)
    q, s = F8.quantize_fp8_blockwise(x)
    back = F8.dequantize_fp8_blockwise(q, s)
    assert (back - x).abs().max() <= x.abs().max() * 0.07
    w = _rnd(200, 384, seed=2)
    wq, ws = F8.quantize_fp8_weight_blocks(w)
    assert ws.shape == (2, 3)
    wb = F8.dequantize_fp8_blockwise(wq, ws, 128)
    assert (wb - w).abs().max() <= w.abs().max() * 0.07


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (300, 520, 384), (1024, 2048, 1024), (64, 8192, 8192)])
def test_fp8_gemm_matches_dequantized_oracle(M, N, K):
    x = _rnd(M, K, seed=3, device="cuda").bfloat16()
    w = _rnd(N, K, seed=4, scale=0.05, device="cuda")
    wq, ws = F8.quantize_fp8_weight_blocks(w)
    aq, sa = F8.quantize_fp8_blockwise(x)  # CUDA quantiser kernel
    aq_ref, sa_ref = F8.quantize_fp8_blockwise(x.cpu())
    torch.testing.assert_close(sa.cpu(), sa_ref, rtol=1e-6, atol=0)
    assert (aq.cpu().float() - aq_ref.float()).abs().max() <= 32  # at most one e4m3 step apart
    res = _rnd(M, N, seed=5, device="cuda").bfloat16()
    out = F8.fp8_gemm_blockscaled(aq, sa, wq, ws, residual=res)
    ref = F8.dequantize_fp8_blockwise(aq.cpu(), sa.cpu()) @ F8.dequantize_fp8_blockwise(wq.cpu(), ws.cpu(), 128).t()
    ref = ref + res.cpu().float()
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), ref, rtol=2e-2, atol=2e-2 * (K / 128) ** 0.5)
    from brain_b200 import _native
    assert _native.status("fp8")[0] == 0


def test_int_group_quant_and_qlinear():
    x = _rnd(8, 256, seed=6)
    q, s, z = Q.quantize_tensor(x, Q.QuantDType.INT8, True, Q.QuantScheme.GROUP_WISE, group_size=64)
    back = Q.dequantize_tensor(q, s, z, x.shape, Q.QuantScheme.GROUP_WISE)
    assert (back - x).abs().max() < x.abs().max() / 100
    q4, s4, z4 = Q.quantize_tensor(x, Q.QuantDType.INT4, True, Q.QuantScheme.GROUP_WISE, group_size=32)
    packed = Q.pack_int4(q4.reshape(-1))
    assert packed.numel() == q4.numel() // 2
    assert torch.equal(Q.unpack_int4(packed, q4.numel()), q4.reshape(-1))
    lin = torch.nn.Linear(256, 32)
    ql = Q.QLinear(lin)
    torch.testing.assert_close(ql(x), lin(x).detach(), rtol=0.05, atol=0.05)
    qa = Q.QLinear(lin, act_quant=True)
    torch.testing.assert_close(qa(x), lin(x).detach(), rtol=0.1, atol=0.1)
    xs = x.clone().requires_grad_(True)
    Q.fake_quantize(xs, torch.tensor(0.05)).sum().backward()
    assert torch.equal(xs.grad, torch.ones_like(x))  # straight-through estimator
    w = _rnd(16, 16, seed=7)
    m = Q.magnitude_prune_(w, 0.5)
    assert int(m.sum()) == 128 and int((w == 0).sum()) == 128


def test_fp8_rowwise_roundtrip_cpu():
    x = _rnd(40, 200, seed=8)
    q, s = F8.quantize_fp8_rowwise(x)
    assert s.shape == (40,)
    assert torch.allclose(s, x.abs().amax(1) / 448.0)
    back = q.float() * s[:, None]
    assert ((back - x).abs() <= x.abs().amax(1, keepdim=True) * 0.07).all()
    z, sz = F8.quantize_fp8_rowwise(torch.zeros(3, 16))
    assert torch.equal(sz, torch.ones(3)) and torch.equal(z.float(), torch.zeros(3, 16))
    w = _rnd(24, 200, seed=9, scale=0.1)
    wq, ws = F8.quantize_fp8_rowwise(w)
    out = F8.fp8_gemm_rowwise(q, s, wq, ws, residual=torch.ones(40, 24))
    ref = (q.float() * s[:, None]) @ (wq.float() * ws[:, None]).t() + 1
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,res", [(512, 768, 512, False),     # CTA-pair kernel, whole tiles
                                       (300, 520, 4096, True),     # pair kernel, ragged M and N, residual
                                       (100, 203, 160, True),      # single-CTA kernel, K tail, N % 8 != 0
                                       (64, 8192, 1024, False)])   # single-CTA kernel (M < 256)
def test_fp8_rowwise_gemm_matches_fp32_oracle(M, N, K, res):
    x = _rnd(M, K, seed=10, device="cuda").bfloat16()
    w = _rnd(N, K, seed=11, scale=0.05, device="cuda").bfloat16()
    aq, sa = F8.quantize_fp8_rowwise(x)  # CUDA quantiser kernel
    aq_ref, sa_ref = F8.quantize_fp8_rowwise(x.cpu())
    torch.testing.assert_close(sa.cpu(), sa_ref, rtol=1e-6, atol=0)
    assert (aq.cpu().float() - aq_ref.float()).abs().max() <= 32  # at most one e4m3 step apart
    wq, ws = F8.quantize_fp8_rowwise(w)
    r = _rnd(M, N, seed=12, device="cuda").bfloat16() if res else None
    out = F8.fp8_gemm_rowwise(aq, sa, wq, ws, residual=r)
    ref = (aq.cpu().float() * sa.cpu()[:, None]) @ (wq.cpu().float() * ws.cpu()[:, None]).t()
    if res:
        ref = ref + r.cpu().float()
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), ref, rtol=2e-2, atol=2e-2 * (K / 128) ** 0.5)
    from brain_b200 import _native
    assert _native.status("fp8")[0] == 0 and _native.status("gemm")[0] == 0
    # against the unquantised bf16 product: the row-wise fp8 error stays within a few percent
    exact = x.float() @ w.float().t() + (r.float() if res else 0)
    rel = float((out.float() - exact).norm() / exact.norm())
    assert rel < 0.05, rel


@pytest.mark.parametrize("scaling", ["rowwise", "block"])
def test_fp8_linear_module_cpu(scaling):
    torch.manual_seed(13)
    lin = torch.nn.Linear(256, 384)
    f = F8.Fp8Linear.from_linear(lin, scaling)
    x = torch.randn(5, 7, 256)
    y = f(x)
    ref = lin(x).detach()
    assert y.shape == (5, 7, 384)
    rel = float((y.float() - ref).norm() / ref.norm())
    assert rel < 0.05, rel
    with pytest.raises(ValueError):
        F8.Fp8Linear(f.wq, f.ws, None, "tensor")


@pytest.mark.gpu
def test_fp8_linear_module_cuda_matches_cpu_oracle():
    torch.manual_seed(14)
    lin = torch.nn.Linear(512, 768).cuda()
    f = F8.Fp8Linear.from_linear(lin, "rowwise")
    x = torch.randn(3, 100, 512, device="cuda")
    y = f(x)
    ref = lin(x).detach()
    rel = float((y.float() - ref).norm() / ref.norm())
    assert rel < 0.05, rel
