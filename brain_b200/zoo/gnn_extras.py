"""Graph construction, datasets, dense/sparse graph operators, a gated convolution, edge models, saliency
explanations, graph batching and a node-classification trainer.

Reference: crates/brain-gnn/src/utils.rs (knn_graph, radius_graph, add_self_loops, random_graph_er),
ops.rs (normalize_adj, sparse_softmax, aggregate_mean/sum/max), graph/ops.rs (in/out degrees,
to_dense_adj, normalized_graph_adj, induced_subgraph), graph/sampler.rs (collate_graphs), layers/gated.rs
(GatedConv), models/edge_model.rs (EdgeClassifier, EdgeRegressor), explain.rs
(saliency_node_importance), datasets/mod.rs (DatasetSplits, random_community_graph, cycle_graph,
zachary_karate_club), train/mod.rs (GnnTrainer).

Everything works on edge-index tensors on the graph's device: distances for k-NN and radius graphs
are one ``cdist``, per-destination softmax and aggregations are scatter reductions, random graphs
draw the reference's LCG stream for all node pairs at once. The reference's ``GnnTrainer`` reports a
surrogate loss without changing the model; this one takes AdamW steps on the masked cross-entropy.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from ..nn.layers import Linear
from ..nn.module import Module
from ..utils.random import lcg64_unit
from .gnn import Graph, scatter_sum


# ------------------------------------------------------------------------------------------ construction
def knn_graph(features: torch.Tensor, k: int) -> torch.Tensor:
    """Edges i -> j to the k nearest other nodes of each i (Euclidean; ties keep the lower index), as
    edge_index [2, n k]."""
    x = features.double().reshape(features.shape[0], -1)
    n = x.shape[0]
    d = torch.cdist(x, x)
    d.fill_diagonal_(float("inf"))
    k = min(k, n - 1)
    order = torch.sort(d, dim=1, stable=True).indices[:, :k]
    src = torch.arange(n, device=x.device).repeat_interleave(k)
    return torch.stack([src, order.reshape(-1)])


def radius_graph(features: torch.Tensor, r: float) -> torch.Tensor:
    """Edges i -> j for every j != i within distance r, ordered by (i, j)."""
    x = features.double().reshape(features.shape[0], -1)
    d = torch.cdist(x, x)
    m = d <= r
    m.fill_diagonal_(False)
    return m.nonzero().t().contiguous()


def add_self_loops(edge_index: torch.Tensor, num_nodes: int) -> torch.Tensor:
    loops = torch.arange(num_nodes, device=edge_index.device).repeat(2, 1)
    return torch.cat([edge_index, loops], 1)


def _pairs(n: int):
    ii, jj = np.meshgrid(np.arange(n), np.arange(n), indexing="ij")
    keep = ii != jj
    return ii[keep], jj[keep]  # row-major order of the ordered pairs i != j


def random_graph_er(n: int, p: float, seed: int) -> torch.Tensor:
    """Erdos-Renyi directed graph: ordered pairs (i, j), i != j, in row-major order each draw one LCG
    uniform from the stream seeded with ``seed``; the edge exists when the draw is below p."""
    i, j = _pairs(n)
    u = lcg64_unit(seed, len(i))
    keep = u < p
    return torch.from_numpy(np.stack([i[keep], j[keep]])).long()


def to_dense_adj(edge_index: torch.Tensor, num_nodes: int, edge_weight=None) -> torch.Tensor:
    """A[s, d] = sum of the weights of edges s -> d (1 each when unweighted)."""
    a = torch.zeros(num_nodes, num_nodes, dtype=torch.float64, device=edge_index.device)
    w = torch.ones(edge_index.shape[1], dtype=torch.float64, device=edge_index.device) if edge_weight is None \
        else edge_weight.double()
    return a.index_put_((edge_index[0], edge_index[1]), w, accumulate=True)


def normalize_adj(adj: torch.Tensor) -> torch.Tensor:
    """D^-1/2 A D^-1/2 with D the row sums (rows of zero degree stay zero)."""
    deg = adj.sum(1)
    inv = torch.where(deg > 0, deg.clamp_min(1e-300).rsqrt(), torch.zeros_like(deg))
    return inv[:, None] * adj * inv[None, :]


def normalized_graph_adj(g: Graph) -> torch.Tensor:
    return normalize_adj(to_dense_adj(g.edge_index, g.num_nodes))


def in_degrees(g: Graph) -> torch.Tensor:
    return torch.bincount(g.edge_index[1], minlength=g.num_nodes)


def out_degrees(g: Graph) -> torch.Tensor:
    return torch.bincount(g.edge_index[0], minlength=g.num_nodes)


def induced_subgraph(g: Graph, nodes, features: torch.Tensor | None = None):
    """The edges with both ends in ``nodes``, renumbered by position in ``nodes``; with node features,
    also their rows in that order."""
    nodes = torch.as_tensor(nodes, dtype=torch.long, device=g.edge_index.device)
    new_id = torch.full((g.num_nodes,), -1, dtype=torch.long, device=nodes.device)
    new_id[nodes] = torch.arange(nodes.numel(), device=nodes.device)
    s, d = new_id[g.edge_index[0]], new_id[g.edge_index[1]]
    keep = (s >= 0) & (d >= 0)
    sub = Graph(torch.stack([s[keep], d[keep]]), nodes.numel())
    return (sub, features[nodes]) if features is not None else sub


def sparse_softmax(scores: torch.Tensor, dst: torch.Tensor, num_nodes: int) -> torch.Tensor:
    """Softmax of edge scores over the edges that share a destination (max-subtracted per destination)."""
    s = scores.double()
    mx = torch.full((num_nodes,), float("-inf"), dtype=s.dtype, device=s.device)
    mx = mx.scatter_reduce(0, dst, s, "amax")
    e = torch.exp(s - torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))[dst])
    tot = torch.zeros(num_nodes, dtype=s.dtype, device=s.device).index_add_(0, dst, e)
    return torch.where(tot[dst] > 0, e / tot[dst].clamp_min(1e-300), torch.zeros_like(e))


def aggregate(edge_features: torch.Tensor, dst: torch.Tensor, num_nodes: int, kind: str = "sum") -> torch.Tensor:
    """Per-destination sum, mean (over the incoming edges) or max (0 for nodes without edges) of edge rows."""
    x = edge_features.reshape(edge_features.shape[0], -1)
    if kind == "sum":
        return scatter_sum(x, dst, num_nodes)
    if kind == "mean":
        cnt = torch.bincount(dst, minlength=num_nodes).clamp_min(1).to(x.dtype)
        return scatter_sum(x, dst, num_nodes) / cnt[:, None]
    if kind == "max":
        out = x.new_full((num_nodes, x.shape[1]), float("-inf"))
        out = out.scatter_reduce(0, dst[:, None].expand_as(x), x, "amax")
        seen = torch.bincount(dst, minlength=num_nodes) > 0
        return torch.where(seen[:, None], out, torch.zeros_like(out))
    raise ValueError(f"unknown aggregation {kind}")


# ------------------------------------------------------------------------------------------ datasets
@dataclass
class DatasetSplits:
    train_mask: torch.Tensor
    val_mask: torch.Tensor
    test_mask: torch.Tensor

    @classmethod
    def new(cls, num_nodes: int, train_ratio: float, val_ratio: float) -> "DatasetSplits":
        """The first floor(n train_ratio) nodes train, the next floor(n val_ratio) validate, the rest test."""
        nt, nv = int(num_nodes * train_ratio), int(num_nodes * val_ratio)
        i = torch.arange(num_nodes)
        return cls(i < nt, (i >= nt) & (i < nt + nv), i >= nt + nv)


def random_community_graph(num_nodes: int, num_communities: int, seed: int):
    """Planted partition: node i is in community i mod c; ordered pairs connect with probability 0.4
    inside a community and 0.05 across (one LCG draw per pair, row-major), then 16 features per node:
    1 at position c mod 16, else 0.1 times the next draw. Returns (graph, features, labels)."""
    c = max(num_communities, 1)
    labels = torch.arange(num_nodes) % c
    i, j = _pairs(num_nodes)
    u = lcg64_unit(seed, len(i) + num_nodes * 15)
    lab = labels.numpy()
    p = np.where(lab[i] == lab[j], 0.4, 0.05)
    keep = u[:len(i)] < p
    g = Graph(torch.from_numpy(np.stack([i[keep], j[keep]])).long(), num_nodes)
    # each node then takes 15 draws for its 15 non-one-hot positions, in position order
    draws = torch.from_numpy(u[len(i):].reshape(num_nodes, 15).copy())
    hot = (labels % 16)[:, None]
    d = torch.arange(16)[None, :]
    feats = 0.1 * draws.gather(1, (d - (d > hot).long()).clamp(0, 14))
    feats[torch.arange(num_nodes), hot[:, 0]] = 1.0
    return g, feats, labels


def cycle_graph(num_nodes: int) -> Graph:
    """Edges i -> i+1 and back, for every i (mod n)."""
    i = torch.arange(num_nodes)
    nx = (i + 1) % num_nodes
    return Graph(torch.stack([torch.stack([i, nx], 1).reshape(-1), torch.stack([nx, i], 1).reshape(-1)]), num_nodes)


_KARATE = [(0, 1), (0, 2), (0, 3), (0, 4), (0, 5), (0, 6), (0, 7), (0, 8), (0, 10), (0, 11), (0, 12), (0, 13),
           (0, 17), (0, 19), (0, 21), (0, 31), (1, 2), (1, 3), (1, 7), (1, 13), (1, 17), (1, 19), (1, 21), (1, 30),
           (2, 3), (2, 7), (2, 8), (2, 9), (2, 13), (2, 27), (2, 28), (2, 32), (3, 7), (3, 12), (3, 13), (4, 6),
           (4, 10), (5, 6), (5, 10), (5, 16), (6, 16), (8, 30), (8, 32), (8, 33), (9, 33), (13, 33), (14, 32),
           (14, 33), (15, 32), (15, 33), (18, 32), (18, 33), (19, 33), (20, 32), (20, 33), (22, 32), (22, 33),
           (23, 25), (23, 27), (23, 29), (23, 32), (23, 33), (24, 25), (24, 27), (24, 31), (25, 31), (26, 29),
           (26, 33), (27, 33), (28, 31), (28, 33), (29, 32), (29, 33), (30, 32), (30, 33), (31, 32), (31, 33),
           (32, 33)]


def zachary_karate_club():
    """Zachary's 34-member karate club (Zachary 1977, 78 friendships, both directions), constant
    features [34, 4] of ones and the reference's labels (members 0-16 class 0, the rest class 1)."""
    g = Graph.from_undirected(_KARATE, 34)
    return g, torch.ones(34, 4, dtype=torch.float64), (torch.arange(34) >= 17).long()


# ------------------------------------------------------------------------------------------ layers / models
class GatedConv(Module):
    """out = (W_t x) * sigmoid(W_g mean_{in-edges} x)."""

    def __init__(self, in_dim: int, out_dim: int, device=None, dtype=None):
        super().__init__()
        self.gate = Linear(in_dim, out_dim, False, device, dtype)
        self.transform = Linear(in_dim, out_dim, False, device, dtype)

    def forward(self, g: Graph, x: torch.Tensor) -> torch.Tensor:
        src, dst = g.edge_index
        agg = aggregate(x[src], dst, g.num_nodes, "mean")
        return self.transform(x) * torch.sigmoid(self.gate(agg))


class EdgeClassifier(Module):
    """Edge logits from the concatenated endpoint embeddings [h_src, h_dst] through one linear map."""

    def __init__(self, node_dim: int, num_classes: int, device=None, dtype=None):
        super().__init__()
        self.lin = Linear(2 * node_dim, num_classes, False, device, dtype)

    def forward(self, g: Graph, h: torch.Tensor) -> torch.Tensor:
        return self.lin(torch.cat([h[g.edge_index[0]], h[g.edge_index[1]]], 1))

    predict_logits = forward


class EdgeRegressor(EdgeClassifier):
    def __init__(self, node_dim: int, device=None, dtype=None):
        super().__init__(node_dim, 1, device, dtype)

    def predict(self, g: Graph, h: torch.Tensor) -> torch.Tensor:
        return self.forward(g, h)


@dataclass
class ExplanationReport:
    node_importance: torch.Tensor
    edge_importance: torch.Tensor

    def top_nodes(self, k: int) -> list[int]:
        return torch.sort(self.node_importance, descending=True, stable=True).indices[:k].tolist()


def saliency_node_importance(g: Graph, embeddings: torch.Tensor) -> ExplanationReport:
    """Node score = L2 norm of its embedding; edge score = mean of its endpoints' scores."""
    ns = embeddings.double().reshape(g.num_nodes, -1).norm(dim=1)
    return ExplanationReport(ns, (ns[g.edge_index[0]] + ns[g.edge_index[1]]) / 2.0)


@dataclass
class BatchGraph:
    """Disjoint union of graphs: node ids offset per graph, ``batch`` maps each node to its graph."""
    graph: Graph
    batch: torch.Tensor
    num_graphs: int


def collate_graphs(graphs) -> BatchGraph:
    edges, batch, off = [], [], 0
    for k, g in enumerate(graphs):
        edges.append(g.edge_index + off)
        batch.append(torch.full((g.num_nodes,), k, dtype=torch.long, device=g.edge_index.device))
        off += g.num_nodes
    ei = torch.cat(edges, 1) if edges else torch.zeros(2, 0, dtype=torch.long)
    return BatchGraph(Graph(ei, off), torch.cat(batch) if batch else torch.zeros(0, dtype=torch.long), len(graphs))


# ------------------------------------------------------------------------------------------ training
@dataclass
class GnnTrainConfig:
    learning_rate: float = 0.01
    weight_decay: float = 1e-4
    num_epochs: int = 10


@dataclass
class GnnTrainStats:
    epoch: int
    train_loss: float
    train_acc: float
    val_loss: float
    val_acc: float


class GnnTrainer:
    """Full-graph node classification: ``model(graph, features)`` gives logits; each epoch is one AdamW
    step on the cross-entropy over the training mask, then loss and accuracy on both masks."""

    def __init__(self, model, config: GnnTrainConfig | None = None):
        self.model, self.c = model, config or GnnTrainConfig()
        self.opt = torch.optim.AdamW(model.parameters(), lr=self.c.learning_rate, weight_decay=self.c.weight_decay)

    def fit(self, g: Graph, x: torch.Tensor, labels: torch.Tensor, splits: DatasetSplits) -> list[GnnTrainStats]:
        stats = []
        for ep in range(self.c.num_epochs):
            logits = self.model(g, x)
            loss = F.cross_entropy(logits[splits.train_mask], labels[splits.train_mask])
            self.opt.zero_grad()
            loss.backward()
            self.opt.step()
            with torch.no_grad():
                logits = self.model(g, x)
                pred = logits.argmax(1)

                def part(m):
                    if not bool(m.any()):
                        return 0.0, 0.0
                    return float(F.cross_entropy(logits[m], labels[m])), float((pred[m] == labels[m]).double().mean())

                tl, ta = part(splits.train_mask)
                vl, va = part(splits.val_mask)
            stats.append(GnnTrainStats(ep, tl, ta, vl, va))
        return stats
