"""Graph construction, datasets, operators, gated convolution, edge models, saliency, batching and the
node-classification trainer against restatements of crates/brain-gnn/src (utils.rs, ops.rs,
graph/ops.rs, datasets/mod.rs, layers/gated.rs, models/edge_model.rs, explain.rs, train/mod.rs)."""
import math

import pytest
import torch

from brain_b200.zoo import gnn_extras as GX
from brain_b200.zoo.gnn import GcnLayer, Graph

M64 = (1 << 64) - 1


def _lcg_units(seed, n):
    s, out = seed, []
    for _ in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & M64
        out.append((s >> 11) / float(1 << 53))
    return out


def test_knn_radius_and_random_graphs():
    x = torch.tensor([[0.0, 0.0], [1.0, 0.0], [0.0, 2.0], [5.0, 5.0]])
    e = GX.knn_graph(x, 2)
    assert e[:, :2].tolist() == [[0, 0], [1, 2]] and e.shape == (2, 8)
    r = GX.radius_graph(x, 2.0)
    assert r.t().tolist() == [[0, 1], [0, 2], [1, 0], [2, 0]]
    er = GX.random_graph_er(6, 0.3, 11)
    u = _lcg_units(11, 30)
    pairs = [(i, j) for i in range(6) for j in range(6) if i != j]
    want = [p for p, v in zip(pairs, u) if v < 0.3]
    assert er.t().tolist() == [list(p) for p in want]
    assert GX.add_self_loops(er, 6).shape[1] == er.shape[1] + 6


def test_dense_ops_softmax_aggregations_subgraph():
    g = Graph(torch.tensor([[0, 1, 1, 2, 2], [1, 0, 2, 1, 1]]), 4)
    a = GX.to_dense_adj(g.edge_index, 4)
    assert a[2, 1] == 2.0 and a[3].sum() == 0
    na = GX.normalize_adj(a)
    deg = a.sum(1)
    assert float(na[0, 1]) == pytest.approx(1.0 / math.sqrt(float(deg[0]) * float(deg[1])))
    assert GX.in_degrees(g).tolist() == [1, 3, 1, 0] and GX.out_degrees(g).tolist() == [1, 2, 2, 0]
    sc = torch.tensor([1.0, 2.0, 3.0, 0.5, -1.0])
    sm = GX.sparse_softmax(sc, g.edge_index[1], 4)
    into1 = torch.tensor([1.0, 0.5, -1.0]).exp()  # edges 0, 3 and 4 all point at node 1
    assert float(sm[0]) == pytest.approx(float(into1[0] / into1.sum()))
    assert float(sm[1]) == pytest.approx(1.0)
    feats = torch.arange(10.0).view(5, 2)
    dst = g.edge_index[1]
    torch.testing.assert_close(GX.aggregate(feats, dst, 4, "sum")[1], feats[[0, 3, 4]].sum(0))
    torch.testing.assert_close(GX.aggregate(feats, dst, 4, "mean")[1], feats[[0, 3, 4]].mean(0))
    mx = GX.aggregate(feats, dst, 4, "max")
    torch.testing.assert_close(mx[1], feats[[0, 3, 4]].max(0).values)
    assert mx[3].tolist() == [0.0, 0.0]
    sub, f = GX.induced_subgraph(g, [2, 1], torch.arange(8.0).view(4, 2))
    assert sub.num_nodes == 2 and sorted(sub.edge_index.t().tolist()) == [[0, 1], [0, 1], [1, 0]]
    assert f.tolist() == [[4.0, 5.0], [2.0, 3.0]]


def test_datasets():
    sp = GX.DatasetSplits.new(10, 0.6, 0.2)
    assert sp.train_mask.sum() == 6 and sp.val_mask.sum() == 2 and sp.test_mask.sum() == 2
    g, x, y = GX.random_community_graph(12, 3, 5)
    n_pairs = 12 * 11
    u = _lcg_units(5, n_pairs + 12 * 15)
    pairs = [(i, j) for i in range(12) for j in range(12) if i != j]
    want = [p for p, v in zip(pairs, u) if v < (0.4 if p[0] % 3 == p[1] % 3 else 0.05)]
    assert g.edge_index.t().tolist() == [list(p) for p in want]
    k = n_pairs
    for n in range(12):
        for d in range(16):
            if d == n % 3:
                assert x[n, d] == 1.0
            else:
                assert float(x[n, d]) == pytest.approx(0.1 * u[k])
                k += 1
    assert y.tolist() == [i % 3 for i in range(12)]
    cg = GX.cycle_graph(5)
    assert cg.edge_index.shape == (2, 10) and GX.in_degrees(cg).tolist() == [2] * 5
    kg, kx, ky = GX.zachary_karate_club()
    assert kg.num_nodes == 34 and kg.edge_index.shape[1] == 156 and int(ky.sum()) == 17
    assert GX.in_degrees(kg)[33] == 17 and GX.in_degrees(kg)[0] == 16


def test_gated_conv_edge_models_saliency_collate():
    g = GX.cycle_graph(4)
    x = torch.randn(4, 3)
    gc = GX.GatedConv(3, 5)
    out = gc(g, x)
    agg = GX.aggregate(x[g.edge_index[0]], g.edge_index[1], 4, "mean")
    torch.testing.assert_close(out, gc.transform(x) * torch.sigmoid(gc.gate(agg)))
    ec = GX.EdgeClassifier(3, 2)
    lg = ec(g, x)
    assert lg.shape == (8, 2)
    torch.testing.assert_close(lg[1], ec.lin(torch.cat([x[g.edge_index[0, 1]], x[g.edge_index[1, 1]]])))
    assert GX.EdgeRegressor(3).predict(g, x).shape == (8, 1)
    rep = GX.saliency_node_importance(g, torch.tensor([[3.0, 4.0], [1.0, 0.0], [0.0, 0.0], [0.0, 2.0]]))
    assert rep.node_importance.tolist() == [5.0, 1.0, 0.0, 2.0] and rep.top_nodes(2) == [0, 3]
    assert float(rep.edge_importance[0]) == pytest.approx((5.0 + 1.0) / 2)
    b = GX.collate_graphs([GX.cycle_graph(3), GX.cycle_graph(2)])
    assert b.graph.num_nodes == 5 and b.batch.tolist() == [0, 0, 0, 1, 1] and int(b.graph.edge_index.max()) == 4


def test_gnn_trainer_learns_the_karate_split():
    torch.manual_seed(0)
    g, _, y = GX.zachary_karate_club()
    x = torch.eye(34)

    class Net(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.l1, self.l2 = GcnLayer(34, 16), GcnLayer(16, 2)

        def forward(self, gr, h):
            return self.l2(gr, torch.relu(self.l1(gr, h)))

    splits = GX.DatasetSplits(torch.ones(34, dtype=torch.bool), torch.zeros(34, dtype=torch.bool),
                              torch.zeros(34, dtype=torch.bool))
    stats = GX.GnnTrainer(Net(), GX.GnnTrainConfig(learning_rate=0.05, num_epochs=60)).fit(g, x, y, splits)
    assert stats[-1].train_loss < stats[0].train_loss and stats[-1].train_acc >= 0.9
