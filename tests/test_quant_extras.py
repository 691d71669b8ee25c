"""Quantisation workflow pieces (crates/brain-quantization/src/calibration.rs, quant_static.rs,
quant_dynamic.rs, ops.rs, error_analysis.rs, mixed.rs, qconv.rs, prune/, graph_quant.rs, bench_quant.rs)."""
import math

import pytest
import torch

from brain_b200.quantization import QLinear
from brain_b200.quantization import extras as QX


def test_int8_matmul_exact_and_requantize():
    g = torch.Generator().manual_seed(0)
    a = torch.randint(-127, 128, (32, 64), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (24, 64), generator=g, dtype=torch.int8)
    assert torch.equal(QX.int8_matmul(a, b), (a.int() @ b.int().t()))
    assert torch.equal(QX.int8_matmul(a[:5], b[:3]), a[:5].int() @ b[:3].int().t())  # small shapes: fallback
    acc = torch.tensor([[1000, -2000], [50, 0]], dtype=torch.int32)
    q = QX.requantize_per_channel(acc, 0.01, torch.tensor([0.5, 0.25]), 0.1)
    assert q.tolist() == [[50, -50], [2, 0]] and q.dtype == torch.int8
    assert QX.requantize(torch.tensor([[100000]], dtype=torch.int32), 1.0, 1.0, 1.0).item() == 127


def test_entropy_observer_clips_outliers():
    g = torch.Generator().manual_seed(0)
    obs = QX.EntropyObserver()
    x = torch.randn(20000, generator=g)
    x[0] = 50.0  # one outlier stretches min-max calibration by 10x
    obs.observe(x)
    obs.observe(torch.randn(20000, generator=g) * 0.5)
    t = obs.threshold()
    assert 2.0 < t < 20.0  # well inside the outlier range, beyond the bulk


def test_error_analysis_dynamic_static_mixed():
    torch.manual_seed(0)
    w = torch.randn(64, 128)
    q = torch.round(w / (w.abs().max() / 127)).clamp(-127, 127) * (w.abs().max() / 127)
    rep = QX.analyze_quantization_error(w, q)
    assert 30 < rep.sqnr_db < 50 and rep.max_abs_error <= float(w.abs().max()) / 127 / 2 + 1e-6
    lin = torch.nn.Linear(128, 48)
    x = torch.randn(40, 128)
    with torch.no_grad():
        ref = lin(x)
    yd = QX.DynamicQuantizer(lin)(x)
    assert float((yd - ref).abs().max()) < 0.05 * float(ref.abs().max())
    st = QX.StaticQuantizer(lin)
    for _ in range(3):
        st.calibrate(torch.randn(40, 128))
    st.freeze()
    assert float((st(x) - ref).abs().max()) < 0.1 * float(ref.abs().max())
    plan = QX.MixedPrecisionQuantizer((4, 8), min_sqnr_db=25.0).plan([("a", torch.randn(64, 64)),
                                                                     ("b", torch.randn(4, 64) * torch.logspace(0, 4, 64))])
    assert plan["a"] in (4, 8) and plan["b"] == 8


def test_qconv2d_and_graph_quantizer():
    torch.manual_seed(0)
    conv = torch.nn.Conv2d(3, 8, 3, padding=1, stride=2)
    x = torch.randn(2, 3, 9, 9)
    with torch.no_grad():
        ref = conv(x)
    for aq in (False, True):
        y = QX.QConv2d(conv, act_quant=aq)(x)
        assert y.shape == ref.shape and float((y - ref).abs().max()) < 0.05 * float(ref.abs().max())
    net = torch.nn.Sequential(torch.nn.Conv2d(3, 4, 3), torch.nn.Flatten(), torch.nn.Linear(4 * 7 * 7, 10),
                              torch.nn.ReLU(), torch.nn.Linear(10, 2))
    xin = torch.randn(3, 3, 9, 9)
    before = net(xin)
    done = QX.GraphQuantizer(skip={"4"}).quantize_(net)
    assert done == ["0", "2"] and isinstance(net[2], QLinear) and isinstance(net[4], torch.nn.Linear)
    assert float((net(xin) - before).abs().max()) < 0.05 * float(before.abs().max()) + 1e-3
    rep = QX.quant_bench(lambda t: conv(t), lambda t: QX.QConv2d(conv)(t), x, iters=2)
    assert rep.max_abs_diff < 0.05 * float(ref.abs().max()) and rep.quant_ms > 0


def test_pruning_schedules():
    w = torch.tensor([[3.0, 4.0], [0.1, 0.1], [1.0, 0.0], [0.0, 2.0]])
    keep = QX.StructuredPruner(0.5).prune_(w)
    assert keep.tolist() == [True, False, False, True] and float(w[1].abs().sum()) == 0
    s = QX.IterativePruneSchedule(0.0, 0.8, 100, 200, 10)
    assert s.sparsity_at(50) == 0.0 and s.sparsity_at(300) == 0.8
    assert s.sparsity_at(150) == pytest.approx(0.8 + (0 - 0.8) * 0.5 ** 3)
    assert s.should_prune(120) and not s.should_prune(125)
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(8, 8), torch.nn.Linear(8, 2))
    lt = QX.LotteryTicketSchedule(net, 0.5)
    with torch.no_grad():
        for p in net.parameters():
            p.add_(torch.randn_like(p))
    sp = lt.next_round(net)
    assert sp == pytest.approx(0.5, abs=0.05)
    w0 = net[0].weight
    m = lt.masks["0.weight"]
    assert torch.equal(w0[m], lt.init["0.weight"][m]) and float(w0[~m].abs().sum()) == 0.0


def test_noam_chained_and_loss_landscape():
    from brain_b200.optim import schedulers as S
    from brain_b200.optim.landscape import LossLandscapeConfig, create_filter_normalized_direction, interpolate_1d, loss_surface

    class Opt:
        lr = 1.0

        def get_lr(self):
            return self.lr

        def set_lr(self, v):
            self.lr = v

    o = Opt()
    n = S.NoamLR(o, d_model=512, warmup_steps=100)
    assert n.lr_at(50) == pytest.approx(512 ** -0.5 * 50 * 100 ** -1.5)
    assert n.lr_at(400) == pytest.approx(512 ** -0.5 * 400 ** -0.5)
    o2 = Opt()
    o2.lr = 0.1

    class Half(S.LRScheduler):
        def lr_at(self, step):
            return self.base_lr * 0.5

    ch = S.ChainedScheduler(o2, [Half(o2), Half(o2)])
    assert ch.step() == pytest.approx(0.025) and o2.lr == pytest.approx(0.025)
    w = torch.randn(4, 6)
    d = create_filter_normalized_direction(w, generator=torch.Generator().manual_seed(0))
    torch.testing.assert_close(d.norm(dim=1), w.norm(dim=1))
    assert float(create_filter_normalized_direction(torch.randn(5)).abs().sum()) == 0.0
    dc = create_filter_normalized_direction(w, kind="constant")
    assert float(dc.norm()) == pytest.approx(float(w.norm()), rel=1e-5) and torch.allclose(dc, dc.flatten()[0].expand_as(dc))
    assert torch.equal(interpolate_1d([w], [d], 0.0)[0], w)
    lin = torch.nn.Linear(3, 1)
    x, y = torch.randn(16, 3), torch.randn(16, 1)
    before = [p.detach().clone() for p in lin.parameters()]
    xs, ls = loss_surface(lin, lambda m: torch.nn.functional.mse_loss(m(x), y), LossLandscapeConfig(num_points=5),
                          generator=torch.Generator().manual_seed(1))
    assert ls.shape == (5,) and float(ls[2]) == pytest.approx(float(torch.nn.functional.mse_loss(lin(x), y)))
    assert all(torch.equal(a, b) for a, b in zip(before, lin.parameters()))
    _, _, surf = loss_surface(lin, lambda m: torch.nn.functional.mse_loss(m(x), y), LossLandscapeConfig(num_points=3),
                              two_d=True)
    assert surf.shape == (3, 3)
