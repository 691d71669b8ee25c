"""Every closed-form VJP against torch autograd on the same op (float64)."""
import math

import pytest
import torch
import torch.nn.functional as F

from brain_b200.autograd import vjps as V


def _auto(fn, *xs, g):
    xs = [x.detach().clone().requires_grad_(True) for x in xs]
    y = fn(*xs)
    return torch.autograd.grad(y, xs, g)


def _r(*s, seed=0, pos=False):
    t = torch.randn(*s, generator=torch.Generator().manual_seed(seed), dtype=torch.float64)
    return t.abs() + 0.5 if pos else t


@pytest.mark.parametrize("name,op", [("add", torch.add), ("sub", torch.sub), ("mul", torch.mul), ("div", torch.div),
                                     ("pow", torch.pow)])
def test_binary_vjps_with_broadcast(name, op):
    a, b = _r(3, 4, seed=1, pos=True), _r(1, 4, seed=2, pos=True)
    g = _r(3, 4, seed=3)
    ga, gb = _auto(op, a, b, g=g)
    assert torch.allclose(getattr(V, f"grad_{name}_a")(a, b, g), ga)
    assert torch.allclose(getattr(V, f"grad_{name}_b")(a, b, g), gb)


def test_matmul_and_unary_vjps():
    a, b, g = _r(2, 3, 4, seed=4), _r(2, 4, 5, seed=5), _r(2, 3, 5, seed=6)
    ga, gb = _auto(torch.matmul, a, b, g=g)
    assert torch.allclose(V.grad_matmul_a(a, b, g), ga) and torch.allclose(V.grad_matmul_b(a, b, g), gb)
    x, xp, gx = _r(4, 6, seed=7), _r(4, 6, seed=8, pos=True), _r(4, 6, seed=9)
    for name, fn, inp in [("exp", torch.exp, x), ("log", torch.log, xp), ("sqrt", torch.sqrt, xp),
                          ("relu", torch.relu, x), ("sigmoid", torch.sigmoid, x), ("tanh", torch.tanh, x),
                          ("silu", F.silu, x), ("gelu", lambda t: F.gelu(t, approximate="tanh"), x)]:
        (ref,) = _auto(fn, inp, g=gx)
        assert torch.allclose(getattr(V, f"grad_{name}")(inp, gx), ref), name
    (ref,) = _auto(lambda t: F.leaky_relu(t, 0.2), x, g=gx)
    assert torch.allclose(V.grad_leaky_relu(x, gx, 0.2), ref)
    (ref,) = _auto(lambda t: torch.softmax(t, 0), x, g=gx)
    assert torch.allclose(V.grad_softmax(x, gx, 0), ref)
    (ref,) = _auto(lambda t: torch.log_softmax(t, -1), x, g=gx)
    assert torch.allclose(V.grad_log_softmax(x, gx, -1), ref)


def test_composite_and_loss_vjps():
    x, gamma, beta, g = _r(3, 8, seed=10), _r(8, seed=11), _r(8, seed=12), _r(3, 8, seed=13)
    ref = _auto(lambda t, w, b: F.layer_norm(t, (8,), w, b, 1e-5), x, gamma, beta, g=g)
    got = V.grad_layernorm(x, gamma, g, 1e-5, normalized_dims=1)
    for a, b in zip(got, ref):
        assert torch.allclose(a, b, atol=1e-10)
    xw, gw = _r(12, seed=14), _r(12, seed=15)  # the reference's whole-tensor form
    gm, gb = _r(12, seed=16), _r(12, seed=17)
    ref = _auto(lambda t, w, b: F.layer_norm(t, (12,), w, b, 1e-5), xw, gm, gb, g=gw)
    assert all(torch.allclose(a, b, atol=1e-10) for a, b in zip(V.grad_layernorm(xw, gm, gw, 1e-5), ref))
    q, k, v, go = _r(2, 5, 4, seed=18), _r(2, 6, 4, seed=19), _r(2, 6, 3, seed=20), _r(2, 5, 3, seed=21)
    ref = _auto(lambda a, b, c: torch.softmax(a @ b.transpose(-1, -2) / 2.0, -1) @ c, q, k, v, g=go)
    assert all(torch.allclose(a, b) for a, b in zip(V.grad_scaled_dot_product_attention(q, k, v, go), ref))
    p, t = _r(4, 3, seed=22), _r(4, 3, seed=23)
    (ref,) = _auto(lambda a: F.mse_loss(a, t) * 2.5, p, g=torch.tensor(1.0, dtype=torch.float64))
    assert torch.allclose(V.grad_mse_loss(p, t, 2.5), ref)
    tgt = [2, 0, 1, 2]
    (ref,) = _auto(lambda a: F.cross_entropy(a, torch.tensor(tgt)), p, g=torch.tensor(1.0, dtype=torch.float64))
    assert torch.allclose(V.grad_cross_entropy_logits(p, tgt), ref)
    y = (t > 0).double()
    (ref,) = _auto(lambda a: F.binary_cross_entropy_with_logits(a, y), p, g=torch.tensor(1.0, dtype=torch.float64))
    assert torch.allclose(V.grad_bce_with_logits(p, y), ref)


def test_shape_index_linalg_pool_conv_vjps():
    x = _r(3, 4, 5, seed=24)
    (ref,) = _auto(lambda t: t.sum(1), x, g=_r(3, 5, seed=25))
    assert torch.allclose(V.grad_sum_axis(_r(3, 5, seed=25), x.shape, 1), ref)
    (ref,) = _auto(lambda t: t.mean(2), x, g=_r(3, 4, seed=26))
    assert torch.allclose(V.grad_mean_axis(_r(3, 4, seed=26), x.shape, 2), ref)
    gp = _r(5, 3, 4, seed=27)
    (ref,) = _auto(lambda t: t.permute(2, 0, 1), x, g=gp)
    assert torch.equal(V.grad_permute(gp, (2, 0, 1)), ref)
    assert torch.equal(V.grad_reshape(x.reshape(12, 5), x.shape), x)
    assert torch.equal(V.grad_transpose(x.transpose(0, 2), 0, 2), x)
    assert torch.equal(V.unbroadcast(torch.ones(2, 3, 4), (3, 1)), torch.full((3, 1), 8.0))
    w, idx, ge = _r(6, 3, seed=28), torch.tensor([1, 4, 1, 0]), _r(4, 3, seed=29)
    (ref,) = _auto(lambda t: F.embedding(idx, t), w, g=ge)
    assert torch.allclose(V.grad_embedding(ge, 6, 3, idx), ref)
    a = _r(4, 4, seed=30) + 4 * torch.eye(4, dtype=torch.float64)
    gi = _r(4, 4, seed=31)
    (ref,) = _auto(torch.linalg.inv, a, g=gi)
    assert torch.allclose(V.grad_inv(torch.linalg.inv(a), gi), ref)
    (ref,) = _auto(torch.linalg.det, a, g=torch.tensor(1.5, dtype=torch.float64))
    assert torch.allclose(V.grad_det(a, torch.linalg.det(a), 1.5), ref)
    img = _r(2, 3, 8, 8, seed=32)
    go = _r(2, 3, 4, 4, seed=33)
    (ref,) = _auto(lambda t: F.max_pool2d(t, 2, 2), img, g=go)
    assert torch.allclose(V.grad_max_pool2d(img, go, 2, 2), ref)
    (ref,) = _auto(lambda t: F.avg_pool2d(t, 2), img, g=go)
    assert torch.allclose(V.grad_avg_pool2d(img.shape, go, 2), ref)
    ga = _r(2, 3, 3, 3, seed=34)
    (ref,) = _auto(lambda t: F.adaptive_avg_pool2d(t, 3), img, g=ga)
    assert torch.allclose(V.grad_adaptive_avg_pool2d(img.shape, ga, 3, 3), ref)
    wc = _r(5, 3, 3, 3, seed=35)
    bc = _r(5, seed=36)
    gc = _r(2, 5, 4, 4, seed=37)
    ref = _auto(lambda t, ww, bb: F.conv2d(t, ww, bb, stride=2, padding=1), img, wc, bc, g=gc)
    got = V.grad_conv2d(img, wc, gc, (2, 2), (1, 1))
    assert all(torch.allclose(p_, r_, atol=1e-10) for p_, r_ in zip(got, ref))
    xt, wt = _r(2, 5, 4, 4, seed=38), _r(5, 3, 3, 3, seed=39)
    gt = _r(2, 3, 9, 9, seed=40)
    ref = _auto(lambda t, ww: F.conv_transpose2d(t, ww, stride=2, padding=0), xt, wt, g=gt)
    got = V.grad_conv_transpose2d(xt, wt, gt, (2, 2), (0, 0))
    assert all(torch.allclose(p_, r_, atol=1e-10) for p_, r_ in zip(got, ref))
    xs = _r(6, seed=41)
    assert torch.equal(V.grad_quantize_ste(xs, torch.ones(6, dtype=torch.float64), -0.5, 0.5),
                       ((xs >= -0.5) & (xs <= 0.5)).double())
    sp, db, gs = _r(3, 4, seed=42), _r(4, 2, seed=43), _r(3, 2, seed=44)
    ref = _auto(torch.matmul, sp, db, g=gs)
    got = V.grad_spmm_dense(sp.to_sparse(), db, gs)
    assert torch.allclose(got[0], ref[0]) and torch.allclose(got[1], ref[1])
    z = torch.complex(_r(8, seed=45), _r(8, seed=46))
    gz = torch.complex(_r(8, seed=47), _r(8, seed=48))
    (ref,) = _auto(torch.fft.fft, z, g=gz)
    assert torch.allclose(V.grad_fft1d(gz), ref)


def test_value_setters_and_grad_helpers():
    from brain_b200.autograd import Value, set_grad_enabled, with_enable_grad, grad_of, zero_grad_from, no_grad
    a = Value.from_slice([1.0, 2.0, 3.0], (3,), requires_grad=True).set_name("a")
    b = Value.from_tensor(torch.tensor([0.5, 0.5, 0.5]), requires_grad=True)
    y = (a * b).sum()
    y.backward()
    assert a.name == "a" and torch.equal(grad_of(a), torch.full((3,), 0.5))
    zero_grad_from(y)
    assert a.grad() is None and b.grad() is None
    a.set_data(torch.tensor([4.0, 5.0, 6.0]))
    assert a.to_vec() == [4.0, 5.0, 6.0]
    a.set_requires_grad(False)
    assert not a.requires_grad
    w = Value(torch.tensor([1.0, -1.0, 2.0])).where_cond(torch.tensor([True, False, True]), torch.zeros(3))
    assert w.to_vec() == [1.0, 0.0, 2.0]
    with set_grad_enabled(False):
        assert not torch.is_grad_enabled()
    with no_grad():
        assert with_enable_grad(torch.is_grad_enabled)
    img = Value(torch.randn(1, 2, 6, 6), requires_grad=True)
    assert img.adaptive_avg_pool2d(3).shape == (1, 2, 3, 3) and img.adaptive_max_pool2d(2).shape == (1, 2, 2, 2)
    out = img.conv_transpose2d(torch.randn(2, 3, 3, 3), stride=2)
    assert out.shape == (1, 3, 13, 13)
