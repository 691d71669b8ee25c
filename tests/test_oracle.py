"""The C++ float64 oracle kernels against the PyTorch float64 restatements of the same ops (two
independent statements of each reference definition must agree to float64 rounding)."""
import math

import torch

from brain_b200 import oracle as O
from brain_b200.ops import attention as attn
from brain_b200.ops import norms
from brain_b200.ops import rope as rope_mod
from brain_b200.ops.cross_entropy import cross_entropy_ref


def _r(*shape, seed=0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed), dtype=torch.float64)


def test_gemm_norms_softmax_ce():
    a, b = _r(7, 13, seed=1), _r(5, 13, seed=2)
    torch.testing.assert_close(O.gemm_nt(a, b), a @ b.t(), rtol=1e-12, atol=1e-12)
    x, w, bb = _r(6, 32, seed=3), _r(32, seed=4), _r(32, seed=5)
    torch.testing.assert_close(O.rms_norm(x, w, 1e-6), norms.rms_norm_ref(x, w, 1e-6).double(), rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(O.layer_norm(x, w, bb, 1e-5), torch.nn.functional.layer_norm(x, (32,), w, bb, 1e-5),
                               rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(O.softmax(x), torch.softmax(x, -1), rtol=1e-12, atol=1e-14)
    labels = torch.tensor([0, 5, -100, 31, 2, 7])
    ref = torch.nn.functional.cross_entropy(x, labels, ignore_index=-100)
    assert abs(float(O.cross_entropy(x, labels)) - float(ref)) < 1e-12
    assert abs(float(O.cross_entropy(x, labels)) - float(cross_entropy_ref(x, labels))) < 1e-5


def test_rope_and_attention():
    x = _r(2, 9, 3, 16, seed=6)
    table = rope_mod.rope_table(16, 32, 500000.0).double()
    torch.testing.assert_close(O.rope(x, 500000.0, offset=4), rope_mod.rope_ref(x, table, None, 4), rtol=1e-6,
                               atol=1e-6)
    q, k, v = _r(2, 11, 4, 8, seed=7), _r(2, 17, 2, 8, seed=8), _r(2, 17, 2, 8, seed=9)
    for causal in (False, True):  # bottom-right causal alignment with Sq < Sk
        ref = attn.sdpa_ref(q, k, v, causal)
        torch.testing.assert_close(O.attention(q, k, v, causal), ref.double(), rtol=1e-6, atol=1e-6)
    # a query row that sees one key returns that key's value
    one = O.attention(_r(1, 1, 1, 8, seed=10), k[:1, :1, :1], v[:1, :1, :1], causal=True)
    torch.testing.assert_close(one[0, 0, 0], v[0, 0, 0])
    assert math.isfinite(float(one.sum()))


import pytest  # noqa: E402


@pytest.mark.gpu
def test_gpu_kernels_against_the_float64_oracle():
    """tcgen05 flash attention, the RMSNorm kernel and the cross-entropy kernel (bf16 inputs) against the
    C++ float64 oracle on the same bf16 values."""
    from brain_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    B, S, Hq, Hkv, D = 1, 256, 4, 2, 128
    q = torch.randn(B, S, Hq, D, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, S, Hkv, D, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, S, Hkv, D, device="cuda", generator=g).bfloat16()
    o = ops.flash_attention(q, k, v, causal=True)
    torch.testing.assert_close(o.double().cpu(), O.attention(q, k, v, True), rtol=3e-2, atol=3e-2)
    x = torch.randn(64, 4096, device="cuda", generator=g).bfloat16()
    w = (torch.randn(4096, device="cuda", generator=g) * 0.1 + 1).bfloat16()
    torch.testing.assert_close(ops.rms_norm(x, w, 1e-6).double().cpu(), O.rms_norm(x, w, 1e-6), rtol=2e-2, atol=2e-2)
    logits = torch.randn(32, 1000, device="cuda", generator=g).bfloat16()
    labels = torch.randint(0, 1000, (32,), device="cuda", generator=g)
    assert abs(float(ops.cross_entropy(logits, labels)) - float(O.cross_entropy(logits, labels))) < 1e-3
    assert not ops.check_status()
