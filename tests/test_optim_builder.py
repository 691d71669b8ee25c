"""Fluent optimizer builder and parameter groups: each built optimizer steps like its direct constructor."""
import pytest
import torch

from brain_b200 import optim
from brain_b200.optim import OptimizerBuilder, OptimizerKind, ParamGroup, ParamGroupConfig, GradEntry


def _quad_step(opt, p):
    opt.zero_grad()
    (p ** 2).sum().backward()
    opt.step()


@pytest.mark.parametrize("kind", list(OptimizerKind))
def test_builder_builds_every_kind(kind):
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(8))
    b = OptimizerBuilder()
    b.kind = kind
    opt = b.lr(1e-2).build([p])
    before = p.detach().clone()
    for _ in range(3):
        _quad_step(opt, p)
    assert not torch.equal(before, p.detach())
    assert (p.detach() ** 2).sum() < (before ** 2).sum()


def test_builder_matches_direct_constructor():
    torch.manual_seed(1)
    p1 = torch.nn.Parameter(torch.randn(16))
    p2 = torch.nn.Parameter(p1.detach().clone())
    a = OptimizerBuilder().adamw().lr(3e-3).betas(0.8, 0.95).weight_decay(0.1).eps(1e-6).build([p1])
    b = optim.AdamW([p2], lr=3e-3, betas=(0.8, 0.95), weight_decay=0.1, eps=1e-6)
    for _ in range(4):
        _quad_step(a, p1)
        _quad_step(b, p2)
    assert torch.equal(p1.detach(), p2.detach())
    lion = OptimizerBuilder().lion()
    assert (lion.beta1, lion.beta2) == (0.9, 0.99)
    sgd = OptimizerBuilder().sgd().momentum(0.9).nesterov(True).build([torch.nn.Parameter(torch.ones(2))])
    assert sgd.param_groups[0]["nesterov"] and sgd.param_groups[0]["momentum"] == 0.9


def test_param_groups_multiplier_and_freeze():
    w = torch.nn.Parameter(torch.ones(4))
    f = torch.nn.Parameter(torch.ones(4))
    g1 = ParamGroup([w], lr=0.1, lr_multiplier=0.5).with_name("body").with_betas(0.9, 0.99).with_weight_decay(0.0)
    g2 = ParamGroup.from_config([f], ParamGroupConfig(name="frozen", lr=0.1, is_frozen=True))
    assert g1.effective_lr() == pytest.approx(0.05) and g2.effective_lr() == 0.0 and g2.initial_lr == 0.1
    opt = OptimizerBuilder().sgd().add_param_group(g1).add_param_group(g2).build()
    opt.zero_grad()
    (w.sum() + f.sum()).backward()
    opt.step()
    assert torch.allclose(w.detach(), torch.full((4,), 0.95)) and torch.equal(f.detach(), torch.ones(4))
    assert [g["name"] for g in opt.param_groups] == ["body", "frozen"]
    assert g1.with_option("momentum_decay", 0.1).options == {"momentum_decay": 0.1}


def test_grad_entry_and_aliases():
    e = GradEntry(3, torch.tensor([3.0, 4.0]))
    assert e.param_id == 3 and e.norm == pytest.approx(5.0) and not e.has_nan
    assert GradEntry(0, torch.tensor([1.0, float("inf")])).has_nan
    assert optim.Rmsprop is optim.RMSprop and optim.SophiaG is optim.Sophia and optim.ModelEma is optim.EMA
    assert optim.SwAOptimizer is optim.SWA and optim.LrFinder is optim.LRFinder
    s = optim.SgdNesterov([torch.nn.Parameter(torch.ones(2))], lr=0.1)
    assert s.param_groups[0]["nesterov"] and s.param_groups[0]["momentum"] == 0.9
