"""The reference's Python package contract (tests/python/test_{tensor,autograd,nn,optim,integration}.py
of the reference, read as a specification) against ``brain_b200.brain``."""
import pytest

import brain_b200.brain as brain


def test_tensor_contract():
    t = brain.Tensor([1.0, 2.0, 3.0, 4.0], shape=[2, 2])
    assert t.shape == [2, 2] and t.ndim == 2 and t.numel == 4 and t.to_list() == [1.0, 2.0, 3.0, 4.0]
    z, o = brain.zeros([3, 4]), brain.ones([2, 5])
    assert z.shape == [3, 4] and all(v == 0.0 for v in z.to_list()) and o.numel == 10
    assert brain.tensor([5.0, 6.0], shape=[2]).to_list() == [5.0, 6.0]
    with pytest.raises(ValueError):
        brain.Tensor([1.0, 2.0], shape=[3, 3])
    assert brain.Tensor([42.0], shape=[1]).item() == 42.0
    with pytest.raises(ValueError):
        brain.Tensor([1.0, 2.0], shape=[2]).item()
    s = brain.Tensor([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], shape=[2, 3])
    assert s.reshape([3, 2]).shape == [3, 2] and s.reshape([3, 2]).to_list() == [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
    assert s.transpose(0, 1).to_list() == [1.0, 4.0, 2.0, 5.0, 3.0, 6.0]
    r = brain.Tensor([1.0, 2.0, 3.0, 4.0], shape=[4])
    assert r.sum().item() == 10.0 and r.mean().item() == 2.5
    a, b = brain.Tensor([1.0, 2.0, 3.0, 4.0], shape=[2, 2]), brain.Tensor([10.0, 20.0, 30.0, 40.0], shape=[2, 2])
    assert (a + b).to_list() == [11.0, 22.0, 33.0, 44.0] and (b - a).to_list() == [9.0, 18.0, 27.0, 36.0]
    assert (a * b).to_list() == [10.0, 40.0, 90.0, 160.0]
    m = brain.Tensor([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], shape=[2, 3]) @ brain.Tensor([7.0, 8.0, 9.0, 1.0, 2.0, 3.0], shape=[3, 2])
    assert m.shape == [2, 2] and m.to_list() == [31.0, 19.0, 85.0, 55.0]
    import brain_b200
    assert brain_b200.Tensor is brain.Tensor


def test_value_autograd_contract():
    v = brain.Value([1.0, 2.0, 3.0], shape=[3], requires_grad=True)
    assert v.shape == [3] and v.requires_grad and v.grad is None
    x = brain.Value([3.0], shape=[1], requires_grad=True)
    y = x * x + x + x + brain.Value([1.0], shape=[1], requires_grad=False)
    assert y.item() == pytest.approx(16.0)
    y.backward()
    assert x.grad.item() == pytest.approx(8.0)
    a, b = brain.Value([2.0], shape=[1], requires_grad=True), brain.Value([5.0], shape=[1], requires_grad=True)
    out = a * b + a
    out.backward()
    assert (out.item(), a.grad.item(), b.grad.item()) == (12.0, 6.0, 2.0)
    s = brain.Value([0.0], shape=[1], requires_grad=True)
    ys = s.sigmoid()
    ys.backward()
    assert ys.item() == 0.5 and s.grad.item() == pytest.approx(0.25)
    t = brain.Value([0.0], shape=[1], requires_grad=True)
    t.tanh().backward()
    assert t.grad.item() == pytest.approx(1.0)
    p = brain.Value([2.5], shape=[1], requires_grad=True)
    p.relu().backward()
    assert p.grad.item() == 1.0
    A = brain.Value([1.0, 2.0, 3.0, 4.0], shape=[2, 2], requires_grad=True)
    B = brain.Value([0.5, -0.5, 1.0, 2.0], shape=[2, 2], requires_grad=True)
    (A @ B).sum().backward()
    assert A.grad.shape == [2, 2] and B.grad.shape == [2, 2]
    assert A.grad.to_list() == [0.0, 3.0, 0.0, 3.0]  # ones @ B^T


def test_nn_contract():
    lin = brain.nn.Linear(4, 8, bias=True)
    ps = lin.parameters()
    assert len(ps) == 2 and ps[0].shape == [8, 4] and ps[1].shape == [8]
    assert lin.forward(brain.Tensor([1.0] * 8, shape=[2, 4])).shape == [2, 8]
    conv = brain.nn.Conv2d(3, 16, 3, bias=True)
    assert conv.parameters()[0].shape == [16, 3, 3, 3]
    assert conv.forward(brain.ones([1, 3, 8, 8])).shape == [1, 16, 8, 8]
    ln = brain.nn.LayerNorm([4], eps=1e-5)
    assert [p.shape for p in ln.parameters()] == [[4], [4]]
    out = ln.forward(brain.Tensor([1.0, 2.0, 3.0, 4.0], shape=[1, 4]))
    assert out.shape == [1, 4] and out.mean().item() == pytest.approx(0.0, abs=1e-4)
    ce = brain.nn.CrossEntropyLoss().forward(brain.Value([[2.0, 0.0]], requires_grad=True), brain.Tensor([0.0]))
    assert ce.item() == pytest.approx(0.126928, abs=1e-5)


@pytest.mark.parametrize("name,start,target,lr,steps,kw,tol", [
    ("SGD", 10.0, 2.0, 0.05, 80, {"momentum": 0.0}, 0.005),
    ("Adam", 8.0, 2.0, 0.1, 200, {}, 0.05),
    ("AdamW", 5.0, 1.0, 0.08, 180, {"weight_decay": 0.001}, 0.05)])
def test_optim_contract(name, start, target, lr, steps, kw, tol):
    w = brain.Value([start], shape=[1], requires_grad=True)
    opt = getattr(brain.optim, name)([w], lr=lr, **kw)
    for _ in range(steps):
        opt.zero_grad()
        loss = w * brain.Value([1.0], requires_grad=False) - brain.Value([target], requires_grad=False)
        loss = loss * loss
        loss.backward()
        opt.step()
    assert abs(w.item() - target) < tol
    w2 = brain.Value([3.0], shape=[1], requires_grad=True)
    o2 = brain.optim.SGD([w2], lr=0.1)
    (w2 * w2).backward()
    assert w2.grad.item() == pytest.approx(6.0)
    o2.zero_grad()
    assert w2.grad is None


def test_integration_custom_module_training_loop():
    class CustomMLP(brain.nn.Module):
        def __init__(self):
            super().__init__()
            self.w1 = brain.Value([0.5, -0.5, 0.2, 0.8, 0.1, -0.3], shape=[3, 2], requires_grad=True)
            self.b1 = brain.Value([0.0, 0.0], shape=[1, 2], requires_grad=True)
            self.w2 = brain.Value([0.4, 0.6], shape=[2, 1], requires_grad=True)
            self.b2 = brain.Value([0.0], shape=[1, 1], requires_grad=True)

        def forward(self, x):
            return (x @ self.w1 + self.b1).relu() @ self.w2 + self.b2

    model = CustomMLP()
    params = model.parameters()
    assert len(params) == 4
    opt = brain.optim.SGD(params, lr=0.02, momentum=0.0)
    crit = brain.nn.MSELoss()
    x = brain.Value([1.0, 0.5, -1.0], shape=[1, 3], requires_grad=False)
    target = brain.Value([1.5], shape=[1, 1], requires_grad=False)
    losses = []
    for _ in range(50):
        opt.zero_grad()
        loss = crit.forward(model(x), target)
        losses.append(loss.item())
        loss.backward()
        opt.step()
    assert losses[-1] < losses[0] and losses[-1] < 0.05
