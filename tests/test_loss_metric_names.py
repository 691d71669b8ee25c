"""Reference-named loss / metric helpers and dispatch by name."""
import pytest
import torch

from brain_b200 import losses as L, metrics as M


def test_loss_aliases_and_helpers():
    assert L.MAELoss is L.L1Loss and L.SimCLRLoss is L.NTXentLoss and L.CompositeLoss is L.CombinedLoss
    per = torch.tensor([1.0, 2.0, 3.0, 4.0])
    assert float(L.apply_loss_mask(per, torch.tensor([1, 0, 1, 0]))) == 2.0
    assert float(L.apply_loss_mask(per, torch.zeros(4))) == 0.0
    assert L.one_hot_target(torch.tensor([2, 0]), 3).tolist() == [[0, 0, 1], [1, 0, 0]]
    x = torch.tensor([[1000.0, 1000.0], [0.0, 0.0]])
    assert torch.allclose(L.log_sum_exp_2d(x), torch.tensor([1000.0 + 0.6931472, 0.6931472]))
    assert float(L.weighted_average(torch.tensor([1.0, 3.0]), torch.tensor([3.0, 1.0]))) == 1.5
    assert float(L.reduction_apply(per, "sum")) == 10.0 and L.clamp_eps(torch.tensor([0.0, 1.0])).tolist()[0] > 0
    p, t = torch.tensor([0.0, 2.0]), torch.tensor([1.0, 1.0])
    assert float(L.compute_loss("mse", p, t)) == 1.0 and float(L.compute_loss("mae", p, t)) == 1.0
    with pytest.raises(ValueError):
        L.compute_loss("nope", p, t)
    assert "huber" in L.loss_names()


def test_metric_aliases_and_helpers():
    assert M.accuracy_score is M.accuracy and M.rmse_score is M.rmse
    assert M.exact_match_ratio(torch.tensor([[1, 0], [1, 1]]), torch.tensor([[1, 0], [0, 1]])) == 0.5
    pred = torch.tensor([[0, 0], [1, 2]])
    tgt = torch.tensor([[0, 1], [1, 2]])
    miou, acc = M.miou_and_pixel_accuracy(pred, tgt, 3)
    # class 0: inter 1, union 2; class 1: inter 1, union 2; class 2: inter 1, union 1
    assert miou == pytest.approx((0.5 + 0.5 + 1.0) / 3) and acc == 0.75
    assert M.logits_to_predictions(torch.tensor([[0.1, 0.9]])).tolist() == [1]
    assert M.binarize_probs(torch.tensor([0.2, 0.5])).tolist() == [0, 1]
    assert M.topk_indices(torch.tensor([3.0, 1.0, 2.0]), 2).tolist() == [0, 2]
    assert M.stable_divide(1, 0, -1) == -1
    assert M.bin_values_uniform(torch.tensor([0.0, 0.49, 1.0, 2.0]), 4).tolist() == [0, 1, 3, 3]
    assert M.edit_distance_levenshtein("abc", "abd") == 1
    assert M.sentence_bleu("a b c d".split(), ["a b c d".split()]) == pytest.approx(1.0)
    assert M.compute_metric("mae", torch.tensor([1.0, 3.0]), torch.tensor([2.0, 2.0])) == pytest.approx(1.0)
    assert "roc_auc" in M.metric_names()


def test_regularization_names():
    from brain_b200 import regularization as R
    from brain_b200.nn import BatchNorm1d, InstanceNorm1d
    e = R.ElasticNetRegularizer(0.1, 0.5)
    assert float(e([torch.tensor([1.0, -2.0])])) == pytest.approx(0.1 * (0.5 * 3 + 0.25 * 5))
    assert R.ElasticWeightConsolidation is R.EWC and R.apply_mixup is R.mixup
    assert BatchNorm1d(4)(torch.randn(3, 4)).shape == (3, 4)
    assert InstanceNorm1d(2)(torch.randn(1, 2, 5)).shape == (1, 2, 5)
