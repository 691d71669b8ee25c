"""Regularisation extras (crates/brain-regularization/src/dropout/adaptive.rs, perturb.rs, consistency.rs,
dropout_uncertainty.rs, stopping.rs, utils.rs, normalization/, registry.rs, regularizers.rs)."""
import math

import pytest
import torch

from brain_b200 import reg_extras as RX


def test_concrete_dropout_learns_and_matches_form():
    cd = RX.ConcreteDropout(0.2, 0.1)
    assert cd.current_p() == pytest.approx(0.2)
    x = torch.ones(1000)
    y = cd(x, generator=torch.Generator().manual_seed(0))
    assert abs(float(y.mean()) - 1.0) < 0.1  # unbiased in expectation
    y.sum().backward()
    assert cd.logit_p.grad is not None and torch.isfinite(cd.logit_p.grad)
    reg = cd.regularizer(torch.tensor(4.0), 10)
    p = 0.2
    want = 1e-6 * 4.0 / (1 - p) + 1e-5 * 10 * (p * math.log(p) + (1 - p) * math.log(1 - p))
    assert float(reg) == pytest.approx(want, rel=1e-5)
    cd.eval()
    assert torch.equal(cd(x), x)


def test_noise_fgsm_consistency_mc():
    gn = RX.GaussianNoise(0.5)
    y = gn(torch.zeros(20000), generator=torch.Generator().manual_seed(1))
    assert abs(float(y.std()) - 0.5) < 0.02
    gn.eval()
    assert float(gn(torch.zeros(3)).abs().sum()) == 0
    x, g = torch.tensor([1.0, 2.0, 3.0]), torch.tensor([0.5, -2.0, 0.0])
    assert RX.apply_fgsm_perturbation(x, g, 0.1).tolist() == pytest.approx([1.1, 1.9, 3.0])
    lin = torch.nn.Linear(3, 2)
    adv = RX.fgsm_example(lin, torch.nn.functional.cross_entropy, torch.randn(4, 3), torch.tensor([0, 1, 0, 1]), 0.05)
    assert adv.shape == (4, 3)
    assert float(RX.compute_consistency_loss(torch.ones(2, 2), torch.zeros(2, 2), 0.5)) == 0.5
    samples = [torch.tensor([1.0, 2.0]), torch.tensor([3.0, 2.0])]
    r = RX.compute_mc_dropout_statistics(samples)
    assert r.mean.tolist() == [2.0, 2.0] and r.variance.tolist() == [1.0, 0.0]
    net = torch.nn.Sequential(torch.nn.Linear(4, 16), torch.nn.Dropout(0.5), torch.nn.Linear(16, 1)).eval()
    outs = RX.mc_dropout_samples(net, torch.randn(3, 4), 8)
    assert outs.shape == (8, 3, 1) and not net.training and float(outs.std(0).sum()) > 0


def test_stop_policies_welford_norm_wrappers_registry():
    assert RX.StopOnBudget(5).should_stop(5, 0.0) and not RX.StopOnBudget(5).should_stop(4, 0.0)
    sp = RX.StopOnPlateau(2, 0.01)
    assert [sp.should_stop(i, l) for i, l in enumerate([1.0, 0.995, 0.99, 0.5, 0.6, 0.7])] == \
        [False, False, True, False, False, True]
    data = torch.randn(50, 3, dtype=torch.float64)
    a, b = RX.WelfordAccumulator(), RX.WelfordAccumulator()
    for row in data[:20]:
        a.update(row)
    for row in data[20:]:
        b.update(row)
    a.merge(b)
    torch.testing.assert_close(a.mean, data.mean(0))
    torch.testing.assert_close(a.variance(), data.var(0, unbiased=False))
    torch.testing.assert_close(a.variance(True), data.var(0, unbiased=True))
    wn = RX.weight_norm(torch.nn.Linear(4, 3))
    assert hasattr(wn.parametrizations, "weight")
    sn = RX.spectral_norm(torch.nn.Linear(4, 3))
    sn(torch.randn(2, 4))
    assert float(torch.linalg.matrix_norm(sn.weight.detach(), 2)) == pytest.approx(1.0, rel=0.2)
    assert RX.RegRegistry.parse_kind("LayerNorm") == "layer_norm"
    with pytest.raises(ValueError):
        RX.RegRegistry.parse_kind("nope")
    p = [torch.tensor([1.0, -2.0])]
    assert float(RX.WeightedRegularizer("l1", 0.1)(p)) == pytest.approx(0.3)
    st = RX.RegStack().add(RX.WeightedRegularizer("l1", 0.1)).add(RX.WeightedRegularizer("l2", 1.0))
    assert float(st(p)) == pytest.approx(0.3 + 0.5 * 5.0)


def test_metric_robust_adversarial_losses():
    import torch.nn.functional as F

    from brain_b200 import losses as L
    cos = torch.tensor([[0.9, 0.1, -0.2], [0.3, 0.5, 0.0]])
    y = torch.tensor([0, 1])
    s, m = 10.0, 0.3
    want = []
    for r in range(2):
        logits = [s * math.cos(math.acos(float(cos[r, c])) + m) if c == int(y[r]) else s * float(cos[r, c])
                  for c in range(3)]
        want.append(-math.log(math.exp(logits[int(y[r])]) / sum(math.exp(v) for v in logits)))
    assert float(L.ArcFaceLoss(s, m)(cos, y)) == pytest.approx(sum(want) / 2, rel=1e-5)
    a, b = torch.tensor([[1.0, 0.0]]), torch.tensor([[0.0, 1.0]])
    assert float(L.AngularDistanceLoss()(a, b)) == pytest.approx(math.pi / 2)
    assert float(L.CauchyLoss(2.0)(torch.tensor([3.0]), torch.tensor([1.0]))) == pytest.approx(0.5 * 4 * math.log(2.0))
    dr, df = torch.tensor([0.8, 1.2]), torch.tensor([0.1, -0.3])
    assert float(L.LSGANLoss.discriminator_loss(dr, df)) == pytest.approx(
        0.5 * float(((dr - 1) ** 2).mean()) + 0.5 * float((df ** 2).mean()))
    assert float(L.RelativisticLoss.discriminator_loss(dr, df)) == pytest.approx(
        float(F.softplus(-(dr - df.mean())).mean() + F.softplus(df - dr.mean()).mean()))


def test_metric_extras():
    from brain_b200 import metrics as M
    assert M.g_mean_score(8, 9, 1, 2) == pytest.approx(math.sqrt(0.8 * 0.9)) and M.g_mean_score(0, 0, 0, 0) == 0.0
    y = torch.tensor([1.0, 2.0, 4.0, 7.0])
    f = torch.tensor([1.5, 2.5, 3.5, 6.0])
    assert M.mase_score(f, y, 1) == pytest.approx((0.5 + 0.5 + 0.5 + 1.0) / 4 / ((1 + 2 + 3) / 3))
    assert M.forecast_bias(f, y) == pytest.approx(-0.125)
    assert M.meteor_score_lite("a b c".split(), "a b d e".split()) == pytest.approx(
        10 * (2 / 3) * 0.5 / (0.5 + 9 * (2 / 3)))
    assert M.cluster_purity([0, 0, 1, 1, 1], [1, 1, 0, 0, 1]) == pytest.approx(4 / 5)
    tpr, fpr = M.threshold_sweep_roc(torch.tensor([0.9, 0.2, 0.6, 0.4]), torch.tensor([1, 0, 1, 0]), 4)
    assert tpr.tolist() == [1.0, 1.0, 1.0, 0.5, 0.0] and fpr.tolist() == [1.0, 0.5, 0.0, 0.0, 0.0]
    assert M.pr_auc_score(torch.tensor([0.9, 0.8, 0.1]), torch.tensor([1, 1, 0])) == pytest.approx(1.0)
    probs = torch.tensor([[0.8, 0.1, 0.1], [0.1, 0.8, 0.1], [0.1, 0.1, 0.8], [0.6, 0.3, 0.1]])
    assert M.multiclass_roc_auc(probs, torch.tensor([0, 1, 2, 0])) == pytest.approx(1.0)
    rep = M.compute_calibration(torch.tensor([0.95, 0.95, 0.15, 0.15]), torch.tensor([1, 0, 0, 0]), 10)
    assert rep.ece == pytest.approx(0.5 * 0.45 + 0.5 * 0.15) and rep.mce == pytest.approx(0.45)
    ag = M.aggregate_metric_runs([1.0, 2.0, 3.0])
    assert ag.mean == 2.0 and ag.std_dev == pytest.approx(1.0) and ag.ci_95_upper == pytest.approx(2 + 1.96 / math.sqrt(3))
    cr = M.compare_models(0.9, 0.8)
    assert cr.is_model_a_better and cr.relative_gain_pct == pytest.approx(12.5)
    tr = M.MetricTracker()
    tr.update("loss", 1.0, 2)
    tr.update("loss", 4.0, 1)
    assert tr.mean("loss") == pytest.approx(2.0) and math.isnan(tr.mean("x"))
    assert tr.summary()["loss"]["count"] == 3 and tr.summary()["loss"]["max"] == 4.0
    assert "| loss | 2.0000 |" in M.format_markdown_report({"loss": tr.mean("loss")})
    assert M.format_csv_report({"a": 1}) == "metric,value\na,1\n"
    assert M.huber_metric(torch.tensor([0.0, 3.0]), torch.tensor([0.5, 0.0])) == pytest.approx((0.125 + 2.5) / 2)
