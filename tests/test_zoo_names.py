"""Reference-named CV, GNN and federated helpers."""
import pytest
import torch


def test_cv_names():
    from brain_b200.zoo import cv as CV
    assert CV.GhostModule is CV.GhostConv and CV.non_max_suppression is CV.nms
    feat = torch.randn(3, 16, 16)
    boxes = torch.tensor([[0.0, 0.0, 8.0, 8.0]])
    assert torch.allclose(CV.RoIAlign(4)(feat, boxes), CV.roi_align(feat, boxes, 4))
    y0, y1, x0, x1 = CV.sample_cutmix_box(32, 32, 0.75, torch.Generator().manual_seed(0))
    assert 0 <= y0 <= y1 <= 32 and 0 <= x0 <= x1 <= 32 and (y1 - y0) <= 16 and (x1 - x0) <= 16


def test_gnn_models_and_loader():
    from brain_b200.zoo import gnn as GN
    torch.manual_seed(0)
    g = GN.Graph.from_undirected([(0, 1), (1, 2), (2, 3)], 4)
    x = torch.randn(4, 5)
    for cls in (GN.GcnModel, GN.SageModel, GN.GinModel, GN.GatModel):
        m = cls(5, 8, 3)
        assert m.forward_node(g, x).shape == (4, 3) and m.forward_graph(g, x).shape == (1, 3)
        assert m.embed_nodes(g, x).shape[0] == 4
    data = [(GN.Graph.from_undirected([(0, 1)], 2), torch.randn(2, 5), k % 2) for k in range(5)]
    ld = GN.GraphLoader(data, batch_size=2)
    batches = list(ld)
    assert ld.num_batches() == 3 and len(batches) == 3
    bg, xb, yb = batches[0]
    assert bg.num_graphs == 2 and xb.shape == (4, 5) and yb.tolist() == [0, 1] and bg.graph.num_nodes == 4
    out = GN.GcnModel(5, 8, 2).forward_graph(bg.graph, xb, bg.batch, pool="add")
    assert out.shape == (2, 2)
    assert GN.aggregate_sum is GN.scatter_sum


def test_federated_helpers():
    from brain_b200 import federated as F
    s = F.sample_clients(100, 0.1, round_idx=3, seed=1)
    assert len(s) == 10 and s == F.sample_clients(100, 0.1, 3, 1) and s != F.sample_clients(100, 0.1, 4, 1)
    a, b = [torch.tensor([3.0, 4.0])], [torch.tensor([-3.0, -4.0])]
    assert F.l2_norm_delta(a) == 5.0 and F.cosine_similarity_deltas(a, b) == pytest.approx(-1.0)
    assert F.estimate_heterogeneity([a, a]) == pytest.approx(0.0) and F.estimate_heterogeneity([a, b]) == pytest.approx(2.0)
    assert F.scale_delta(a, 2)[0].tolist() == [6.0, 8.0]
    assert F.communication_cost_bytes(1000, 10, 5) == 1000 * 4 * 10 * 5 * 2
    assert F.polyak_average([torch.zeros(1)], [torch.ones(1)], 0.9)[0].item() == pytest.approx(0.1)
    assert F.normalize_weights([1, 3]) == [0.25, 0.75] and F.stddev([1, 3]) == 1.0
    assert F.cosine_lr(0.1, 0, 10) == pytest.approx(0.1) and F.cosine_lr(0.1, 10, 10) == pytest.approx(0.0)
    mon = F.FedMonitor(window=2, tol=1e-3)
    for l in (1.0, 0.5, 0.49999, 0.49998):
        mon.record(l)
    assert mon.latest_loss() == 0.49998 and mon.has_converged()
    model = torch.nn.Linear(2, 1)
    tr = F.LocalTrainer(model, torch.nn.functional.mse_loss, lr=0.1, epochs=2)
    xs = torch.randn(8, 2)
    delta, n = tr.train([(xs, xs.sum(1, keepdim=True))])
    assert n == 8 and len(delta) == 2 and F.l2_norm_delta(delta) > 0


def test_rl_names():
    from brain_b200.zoo import rl_agents as RA, rl as RL
    sch = RA.EpsilonSchedule(1.0, 0.1, 100)
    assert sch.get_epsilon(0) == 1.0 and sch.get_epsilon(50) == pytest.approx(0.55) and sch.get_epsilon(500) == pytest.approx(0.1)
    pol = RA.EpsilonGreedyPolicy(RA.EpsilonSchedule(0.0, 0.0, 1), 4)
    assert pol.select_action(torch.tensor([[0.0, 3.0, 1.0, 2.0]]), 10).tolist() == [1]
    tgt, src = torch.nn.Linear(2, 2), torch.nn.Linear(2, 2)
    before = tgt.weight.detach().clone()
    RA.soft_update_target(tgt, src, 0.5)
    assert torch.allclose(tgt.weight, 0.5 * before + 0.5 * src.weight)
    vt = RA.VTable(3, gamma=0.5, lr=1.0)
    vt.v[2] = 4.0
    assert vt.update_td(0, 1.0, 2, False) == 3.0 and float(vt.v[0]) == 3.0
    st = RA.SumTree(5)
    for i, p in enumerate([1.0, 2.0, 3.0, 4.0, 0.5]):
        st.update(i, p)
    assert st.total_priority() == 10.5
    assert st.get_leaf(0.5)[0] == 0 and st.get_leaf(1.5)[0] == 1 and st.get_leaf(6.2)[0] == 3 and st.get_leaf(10.2)[0] == 4
    ag = RA.make_agent("dqn", 4, 2)
    assert isinstance(ag, RL.DqnAgent) and isinstance(RA.make_agent("ppo", 4, 2), RL.PpoAgent)
    with pytest.raises(ValueError):
        RA.make_agent("nope", 4, 2)
    assert RA.compute_gae is RL.gae and RA.CartPoleEnv is RA._envs.CartPole


def test_train_names():
    from brain_b200 import train as TR
    assert TR.CallbackAction.from_bool(True) == "stop" and TR.CallbackAction.from_bool(False) == "continue"
    assert TR.check_improvement(0.5, None) and TR.check_improvement(0.5, 0.6) and not TR.check_improvement(0.59, 0.6, min_delta=0.05)
    assert TR.check_improvement(0.9, 0.8, mode="max")
    assert TR.argmax_rows([[0.1, 0.9], [0.7, 0.3]]) == [1, 0]
    w = TR.WindowedAverage(2)
    w.update(1.0)
    w.update(3.0)
    assert w.update(5.0) == 4.0
    p = torch.ones(2, requires_grad=True)
    m = TR.TrainableModule(lambda x: x * p, [p])
    assert list(m.parameters())[0] is p and m(torch.tensor([2.0, 3.0])).tolist() == [2.0, 3.0]
    assert TR.L2Regularization is TR.L2Regularizer


def test_mobilenet_v3():
    from brain_b200.zoo.cv_extras import mobilenet_v3, InvertedResidual
    torch.manual_seed(0)
    m = mobilenet_v3(10, "small")
    y = m(torch.randn(2, 3, 64, 64))
    assert y.shape == (2, 10)
    n = sum(p.numel() for p in m.parameters())
    assert 1.3e6 < n < 1.7e6  # the published small variant: about 2.5 M parameters with a 1000-class head
    assert m.forward_features(torch.randn(1, 3, 64, 64)).shape == (1, 576, 2, 2)
    blk = InvertedResidual(16, 3, 64, 16, True, "hs", 1)
    assert blk.residual and blk(torch.randn(1, 16, 8, 8)).shape == (1, 16, 8, 8)
    m.train()
    loss = torch.nn.functional.cross_entropy(m(torch.randn(4, 3, 32, 32)), torch.tensor([0, 1, 2, 3]))
    loss.backward()
    assert all(p.grad is not None for p in m.parameters() if p.requires_grad)
