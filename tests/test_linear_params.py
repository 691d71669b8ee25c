"""LinearParams: the reference's [in, out] projection layout and position-hash initialisation
(crates/brain-transformer/src/core.rs:110-191), conversion to this framework's [out, in] Linear weights,
and the tcgen05 forward on the [in, out] weight."""
import math

import pytest
import torch

from brain_b200.models.linear_params import LinearParams, load_reference_projection, reference_init


def _formula(i, j, seed, fin, fout):
    std = math.sqrt(2.0 / (fin + fout))
    x = math.sin(float(seed + i * 10007 + j * 37 + 1)) * 43758.5453
    return (x - math.trunc(x)) * 2.0 * std - std


def test_init_follows_the_position_hash():
    w = reference_init(16, 32, seed=1, exact=True)
    assert w.shape == (16, 32) and w.dtype == torch.float64
    for i, j in [(0, 0), (3, 7), (15, 31), (9, 0)]:
        assert w[i, j].item() == _formula(i, j, 1, 16, 32)  # bit-exact with the exact path
    fast = reference_init(16, 32, seed=1)
    assert (fast - w).abs().max().item() < 1e-9
    std = math.sqrt(2.0 / 48)
    # fract keeps the sign of sin(s) * 43758.5453, so values span (-3 std, std)
    assert w.max().item() <= std and w.min().item() >= -3 * std and w.std().item() > 0.3 * std
    assert not torch.equal(reference_init(16, 32, seed=2), fast)  # the seed changes the weights


def test_reference_forward_and_shapes():
    lp = LinearParams(16, 32, has_bias=True, seed=1, dtype=torch.float64, exact=True)
    assert lp.weight.shape == (16, 32) and lp.bias.shape == (32,)
    x = torch.ones(2, 4, 16, dtype=torch.float64)
    y = lp(x)
    assert y.shape == (2, 4, 32)
    torch.testing.assert_close(y[0, 0], lp.weight.sum(0))  # ones @ W = column sums, zero bias
    with pytest.raises(ValueError):
        lp(torch.ones(2, 15, dtype=torch.float64))


def test_layout_conversion_round_trip():
    lp = LinearParams(24, 40, has_bias=True, seed=5)
    with torch.no_grad():
        lp.bias.copy_(torch.randn(40))
    lin = torch.nn.Linear(24, 40)
    lp.load_into(lin)
    x = torch.randn(3, 24)
    torch.testing.assert_close(lin(x), lp(x), rtol=1e-5, atol=1e-5)
    back = LinearParams.from_linear_weight(lin.weight.detach(), lin.bias.detach())
    torch.testing.assert_close(back.weight, lp.weight)
    raw = torch.empty(40, 24)
    load_reference_projection(raw, lp.weight.detach())
    torch.testing.assert_close(raw, lp.weight.detach().t())


@pytest.mark.gpu
def test_tcgen05_forward_on_in_out_weight():
    lp = LinearParams(512, 768, has_bias=True, seed=3, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lp.bias.copy_(torch.randn(768, device="cuda"))
    x = torch.randn(4, 64, 512, device="cuda").bfloat16()
    y = lp(x)
    ref = x.float() @ lp.weight.float() + lp.bias.float()
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)
