"""Graph neural networks: a COO ``Graph``, GCN / GraphSAGE / GIN / GAT / EdgeConv layers, global
readouts, a neighbour sampler, and a node-classification model.

Reference: crates/brain-gnn. ``GcnLayer`` (layers/gcn.rs:14-60: symmetric normalisation
D^-1/2 (A + I) D^-1/2), ``GatLayer`` (layers/gat.rs:14-80: multi-head additive attention with
LeakyReLU 0.2 over each node's neighbourhood), ``SageLayer`` (layers/sage.rs: mean aggregator,
concatenated with the node's own features), ``GinLayer`` (layers/gin.rs: MLP((1 + eps) x + Σ neighbours)),
edge convolution (layers/edge_conv.rs), readouts (readout/mod.rs:12-80: add / mean / max pool by graph
id), sampler (graph/sampler.rs).

Message passing is gather + ``index_add_`` (scatter-sum) over the edge list, and the per-layer
feature transforms go through ``brain_b200.nn.Linear``; everything stays on the graph's device.
"""
from __future__ import annotations

import torch

from ..nn.layers import Linear
from ..nn.module import Module


class Graph:
    """Directed edges ``src -> dst`` ([2, E] int64); messages flow from src to dst."""

    def __init__(self, edge_index: torch.Tensor, num_nodes: int):
        self.edge_index = edge_index.long()
        self.num_nodes = num_nodes

    @classmethod
    def from_undirected(cls, edges, num_nodes: int, device=None) -> "Graph":
        e = torch.as_tensor(edges, dtype=torch.long, device=device).reshape(-1, 2).t()
        return cls(torch.cat([e, e.flip(0)], 1), num_nodes)

    def with_self_loops(self) -> "Graph":
        loops = torch.arange(self.num_nodes, device=self.edge_index.device).repeat(2, 1)
        return Graph(torch.cat([self.edge_index, loops], 1), self.num_nodes)

    def in_degree(self) -> torch.Tensor:
        return torch.bincount(self.edge_index[1], minlength=self.num_nodes)

    def neighbors(self, node: int) -> torch.Tensor:
        return self.edge_index[0, self.edge_index[1] == node]


def scatter_sum(msg: torch.Tensor, index: torch.Tensor, n: int) -> torch.Tensor:
    out = msg.new_zeros((n,) + msg.shape[1:])
    return out.index_add_(0, index, msg)


def scatter_max(msg: torch.Tensor, index: torch.Tensor, n: int) -> torch.Tensor:
    out = msg.new_full((n,) + msg.shape[1:], float("-inf"))
    out = out.scatter_reduce(0, index.view(-1, *([1] * (msg.dim() - 1))).expand_as(msg), msg, "amax")
    return torch.where(torch.isinf(out), torch.zeros_like(out), out)


class GcnLayer(Module):
    def __init__(self, in_dim: int, out_dim: int, bias: bool = True, device=None, dtype=None):
        super().__init__()
        self.lin = Linear(in_dim, out_dim, bias, device, dtype)

    def forward_gcn(self, g: Graph, x: torch.Tensor) -> torch.Tensor:
        gl = g.with_self_loops()
        src, dst = gl.edge_index
        deg = gl.in_degree().to(x.dtype)
        norm = deg.rsqrt()[src] * deg.rsqrt()[dst]
        h = self.lin(x)
        return scatter_sum(h[src] * norm[:, None], dst, g.num_nodes)

    forward = forward_gcn


class SageLayer(Module):
    def __init__(self, in_dim: int, out_dim: int, device=None, dtype=None):
        super().__init__()
        self.self_lin = Linear(in_dim, out_dim, True, device, dtype)
        self.nbr_lin = Linear(in_dim, out_dim, False, device, dtype)

    def forward(self, g: Graph, x):
        src, dst = g.edge_index
        deg = g.in_degree().clamp(min=1).to(x.dtype)
        mean = scatter_sum(x[src], dst, g.num_nodes) / deg[:, None]
        return self.self_lin(x) + self.nbr_lin(mean)


class GinLayer(Module):
    def __init__(self, in_dim: int, out_dim: int, eps: float = 0.0, train_eps: bool = True, device=None, dtype=None):
        super().__init__()
        self.eps = torch.nn.Parameter(torch.tensor(float(eps), device=device)) if train_eps else eps
        self.mlp1 = Linear(in_dim, out_dim, True, device, dtype)
        self.mlp2 = Linear(out_dim, out_dim, True, device, dtype)

    def forward(self, g: Graph, x):
        src, dst = g.edge_index
        agg = (1 + self.eps) * x + scatter_sum(x[src], dst, g.num_nodes)
        return self.mlp2(torch.relu(self.mlp1(agg)))


class GatLayer(Module):
    """Per head: e_ij = LeakyReLU(a_src · W x_j + a_dst · W x_i), softmax over the in-edges of i
    (self-loop included), output the α-weighted sum; heads are concatenated (or averaged)."""

    def __init__(self, in_dim: int, out_dim: int, num_heads: int = 1, concat: bool = True, device=None, dtype=None):
        super().__init__()
        self.h, self.d, self.concat = num_heads, out_dim, concat
        self.lin = Linear(in_dim, num_heads * out_dim, False, device, dtype)
        self.a_src = torch.nn.Parameter(torch.randn(num_heads, out_dim, device=device, dtype=dtype) * 0.1)
        self.a_dst = torch.nn.Parameter(torch.randn(num_heads, out_dim, device=device, dtype=dtype) * 0.1)

    def forward_gat(self, g: Graph, x):
        gl = g.with_self_loops()
        src, dst = gl.edge_index
        h = self.lin(x).view(-1, self.h, self.d)
        e = torch.nn.functional.leaky_relu((h[src] * self.a_src).sum(-1) + (h[dst] * self.a_dst).sum(-1), 0.2)
        emax = scatter_max(e, dst, g.num_nodes)
        w = torch.exp(e - emax[dst])
        denom = scatter_sum(w, dst, g.num_nodes)
        alpha = w / denom[dst]
        out = scatter_sum(h[src] * alpha[..., None], dst, g.num_nodes)
        return out.reshape(g.num_nodes, -1) if self.concat else out.mean(1)

    forward = forward_gat


class EdgeConv(Module):
    """x_i' = max_j MLP([x_i, x_j − x_i]) over the in-neighbours j of i (DGCNN)."""

    def __init__(self, in_dim: int, out_dim: int, device=None, dtype=None):
        super().__init__()
        self.lin = Linear(2 * in_dim, out_dim, True, device, dtype)

    def forward(self, g: Graph, x):
        src, dst = g.edge_index
        m = torch.relu(self.lin(torch.cat([x[dst], x[src] - x[dst]], -1)))
        return scatter_max(m, dst, g.num_nodes)


def global_add_pool(x, batch, num_graphs: int):
    return scatter_sum(x, batch, num_graphs)


def global_mean_pool(x, batch, num_graphs: int):
    cnt = torch.bincount(batch, minlength=num_graphs).clamp(min=1).to(x.dtype)
    return scatter_sum(x, batch, num_graphs) / cnt[:, None]


def global_max_pool(x, batch, num_graphs: int):
    return scatter_max(x, batch, num_graphs)


def sample_neighbors(g: Graph, nodes: torch.Tensor, fanout: int, generator=None) -> Graph:
    """Keeps at most ``fanout`` random in-edges for each node of ``nodes`` (GraphSAGE sampling)."""
    src, dst = g.edge_index
    keep = []
    for n in nodes.tolist():
        idx = (dst == n).nonzero().view(-1)
        if idx.numel() > fanout:
            idx = idx[torch.randperm(idx.numel(), generator=generator, device="cpu")[:fanout].to(idx.device)]
        keep.append(idx)
    sel = torch.cat(keep) if keep else torch.zeros(0, dtype=torch.long, device=src.device)
    return Graph(g.edge_index[:, sel], g.num_nodes)


class GnnNodeClassifier(Module):
    def __init__(self, in_dim: int, hidden: int, num_classes: int, layer: str = "gcn", heads: int = 2, device=None,
                 dtype=None):
        super().__init__()
        if layer == "gat":
            self.l1 = GatLayer(in_dim, hidden, heads, True, device, dtype)
            self.l2 = GatLayer(hidden * heads, num_classes, 1, False, device, dtype)
        else:
            cls = {"gcn": GcnLayer, "sage": SageLayer, "gin": GinLayer}[layer]
            self.l1 = cls(in_dim, hidden, device=device, dtype=dtype)
            self.l2 = cls(hidden, num_classes, device=device, dtype=dtype)

    def forward(self, g: Graph, x):
        return self.l2(g, torch.relu(self.l1(g, x)))


class GraphTransformerLayer(Module):
    """Multi-head scaled dot-product attention restricted to each node's in-edges (self-loop added),
    with a residual connection and LayerNorm (reference layers/transformer.rs)."""

    def __init__(self, dim: int, heads: int = 4, device=None, dtype=None):
        super().__init__()
        self.h, self.d = heads, dim // heads
        self.q = Linear(dim, dim, False, device, dtype)
        self.k = Linear(dim, dim, False, device, dtype)
        self.v = Linear(dim, dim, False, device, dtype)
        self.o = Linear(dim, dim, True, device, dtype)
        self.norm = torch.nn.LayerNorm(dim, device=device, dtype=dtype)

    def forward(self, g: Graph, x):
        gl = g.with_self_loops()
        src, dst = gl.edge_index
        N = g.num_nodes
        q, k, v = (f(x).view(N, self.h, self.d) for f in (self.q, self.k, self.v))
        e = (q[dst] * k[src]).sum(-1) / self.d ** 0.5  # [E, H]
        emax = scatter_max(e, dst, N)
        w = torch.exp(e - emax[dst])
        alpha = w / scatter_sum(w, dst, N)[dst]
        out = scatter_sum(v[src] * alpha[..., None], dst, N).reshape(N, -1)
        return self.norm(x + self.o(out))


def jumping_knowledge(layer_outputs, mode: str = "cat"):
    """Combine the node embeddings of every layer: concatenation, element-wise max or mean (JK-Net)."""
    if mode == "cat":
        return torch.cat(layer_outputs, -1)
    st = torch.stack(layer_outputs)
    return st.max(0).values if mode == "max" else st.mean(0)


# ------------------------------------------------------------------ the reference's names
# crates/brain-gnn/src: models/{mod,gin_model}.rs (GcnModel, SageModel, GatModel, GinModel with forward_node /
# forward_graph / embed_nodes), ops.rs (aggregate_sum, aggregate_max), datasets/loader.rs (GraphLoader,
# GraphBatch), readout/jumping.rs (JkMode).
aggregate_sum = scatter_sum
aggregate_max = scatter_max


class _GnnModel(GnnNodeClassifier):
    LAYER = "gcn"

    def __init__(self, in_dim: int, hidden: int, num_classes: int, **kw):
        super().__init__(in_dim, hidden, num_classes, layer=self.LAYER, **kw)

    def forward_node(self, g: Graph, x):
        """Per-node logits."""
        return self.forward(g, x)

    def embed_nodes(self, g: Graph, x):
        """Hidden node embeddings after the first layer."""
        return torch.relu(self.l1(g, x))

    def forward_graph(self, g: Graph, x, batch=None, pool: str = "mean"):
        """Graph-level logits: node logits pooled per graph (``batch`` maps nodes to graphs)."""
        h = self.forward(g, x)
        if batch is None:
            batch = torch.zeros(h.shape[0], dtype=torch.long, device=h.device)
        n = int(batch.max()) + 1 if batch.numel() else 0
        return {"mean": global_mean_pool, "add": global_add_pool, "max": global_max_pool}[pool](h, batch, n)


class GcnModel(_GnnModel):
    LAYER = "gcn"


class SageModel(_GnnModel):
    LAYER = "sage"


class GatModel(_GnnModel):
    LAYER = "gat"


class GinModel(_GnnModel):
    LAYER = "gin"


class JkMode:
    CONCAT, MAX, LAST = "cat", "max", "last"


class GraphLoader:
    """Mini-batches of small graphs, a list of (Graph, node features x, label y): each batch is
    (BatchGraph of the disjoint union, concatenated x, stacked y)."""

    def __init__(self, graphs, batch_size: int, shuffle: bool = False, seed: int = 0):
        self.graphs, self.bs, self.shuffle, self.seed, self.epoch = list(graphs), batch_size, shuffle, seed, 0

    def num_batches(self) -> int:
        return -(-len(self.graphs) // self.bs)

    def get_batch(self, i: int, order=None):
        from .gnn_extras import collate_graphs
        order = order if order is not None else list(range(len(self.graphs)))
        items = [self.graphs[j] for j in order[i * self.bs:(i + 1) * self.bs]]
        bg = collate_graphs([it[0] for it in items])
        return bg, torch.cat([it[1] for it in items]), torch.stack([torch.as_tensor(it[2]) for it in items])

    def __iter__(self):
        order = list(range(len(self.graphs)))
        if self.shuffle:
            order = torch.randperm(len(order), generator=torch.Generator().manual_seed(self.seed + self.epoch)).tolist()
        self.epoch += 1
        for i in range(self.num_batches()):
            yield self.get_batch(i, order)
