"""Graph-IR tooling with the reference's names: a fluent ``GraphBuilder``, model-graph builders (MLP,
CNN-free MLP-mixer style blocks, transformer block), ``compute_topological_order``, level schedules and
parallelism (``generate_schedule`` / ``analyze_parallelism`` / ``max_parallelism``), fusion candidates,
algebraic rewrites (x * 1, x + 0, x - 0, x / 1, identity chains), sub-graph cloning, per-node
profiling, graph summaries and memory totals, and ``ExecutionEngine``: the interpreter's node sequence
captured once into a CUDA graph on GPU (so a whole graph replays as one launch), plain interpretation
on the CPU.

Reference: crates/brain-graph/src/builder.rs (GraphBuilder, add_constant), helper.rs
(build_mlp_graph / build_transformer_graph), topology.rs (compute_topological_order), schedule.rs
(SchedulePlan, generate_schedule, max_parallelism), analyze.rs (analyze_parallelism,
analyze_fusion_candidates, analyze_cycles), transform.rs (rewrite_algebraic), clone.rs (clone_subgraph),
profile.rs (profile_graph, GraphProfile), utils.rs (format_graph_summary), impl_.rs
(total_output_memory_bytes, run_graph); crates/brain-compile/src/exec.rs (ExecutionEngine),
export_ir.rs (export_text), ops.rs (arithmetic_intensity).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from .graph import GraphError, GraphInterpreter, GraphIr, estimate_flops, infer_shapes, plan_fusion, run_op


class GraphBuilder:
    """``b = GraphBuilder("mlp"); x = b.input("x", [B, D]); y = b.op("relu", x); b.output(y); g = b.build()``."""

    def __init__(self, name: str = "graph"):
        self.g = GraphIr(name)

    def input(self, name: str, shape=None, dtype: str = "float32") -> int:
        return self.g.add_input(name, shape, dtype)

    def add_constant(self, name: str, data) -> int:
        return self.g.constant(name, torch.as_tensor(data))

    def op(self, op: str, *inputs, **attrs) -> int:
        return self.g.add_node(op, list(inputs), attrs)

    def output(self, *vids) -> None:
        self.g.mark_output(*vids)

    def build(self) -> GraphIr:
        infer_shapes(self.g)
        return self.g


def build_mlp_graph(dims, act: str = "relu", batch: int = 1, seed: int = 0) -> GraphIr:
    """x [batch, dims[0]] -> linear -> act -> ... -> linear (no act after the last)."""
    g = torch.Generator().manual_seed(seed)
    b = GraphBuilder("mlp")
    h = b.input("x", [batch, dims[0]])
    for i, (di, do) in enumerate(zip(dims[:-1], dims[1:])):
        w = b.add_constant(f"w{i}", torch.randn(do, di, generator=g) * di ** -0.5)
        bias = b.add_constant(f"b{i}", torch.zeros(do))
        h = b.op("linear", h, w, bias)
        if i < len(dims) - 2:
            h = b.op(act, h)
    b.output(h)
    return b.build()


def build_transformer_graph(seq: int, dim: int, ffn: int, seed: int = 0) -> GraphIr:
    """One pre-norm block on x [seq, dim] (single head): LN -> q/k/v linears -> softmax(q k^T / sqrt d) v
    -> out linear -> residual; LN -> SwiGLU FFN -> residual."""
    g = torch.Generator().manual_seed(seed)

    def w(b, name, o, i):
        return b.add_constant(name, torch.randn(o, i, generator=g) * i ** -0.5)
    b = GraphBuilder("transformer_block")
    x = b.input("x", [seq, dim])
    h = b.op("layer_norm", x)
    q, k, v = (b.op("linear", h, w(b, n, dim, dim)) for n in ("wq", "wk", "wv"))
    s = b.op("constant_scale", b.op("matmul", q, b.op("transpose", k)), scale=dim ** -0.5)
    a = b.op("matmul", b.op("softmax", s), v)
    x = b.op("add", x, b.op("linear", a, w(b, "wo", dim, dim)))
    h = b.op("layer_norm", x)
    gu = b.op("linear", h, w(b, "w_gate_up", 2 * ffn, dim))
    x = b.op("add", x, b.op("linear", b.op("swiglu", gu), w(b, "w_down", dim, ffn)))
    b.output(x)
    return b.build()


def compute_topological_order(g: GraphIr) -> list:
    """Nodes ordered so every node follows the producers of its inputs (Kahn's algorithm); raises on a cycle."""
    prod = g.producers()
    deps = {id(n): {id(prod[i]) for i in n.inputs if i in prod} for n in g.nodes}
    by_id = {id(n): n for n in g.nodes}
    ready = [n for n in g.nodes if not deps[id(n)]]
    out, done = [], set()
    users: dict[int, list] = {}
    for n in g.nodes:
        for d in deps[id(n)]:
            users.setdefault(d, []).append(n)
    while ready:
        n = ready.pop(0)
        out.append(n)
        done.add(id(n))
        for u in users.get(id(n), []):
            if id(u) not in done and deps[id(u)] <= done and u not in ready and u not in out:
                ready.append(u)
    if len(out) != len(by_id):
        raise GraphError("cycle in graph")
    return out


@dataclass
class SchedulePlan:
    levels: list = field(default_factory=list)  # nodes that can run concurrently, level by level

    @property
    def max_parallelism(self) -> int:
        return max((len(lv) for lv in self.levels), default=0)

    @property
    def depth(self) -> int:
        return len(self.levels)


def generate_schedule(g: GraphIr) -> SchedulePlan:
    """Level of a node = 1 + max level of its producers (inputs and constants at level -1)."""
    prod = g.producers()
    lvl: dict[int, int] = {}
    levels: list[list] = []
    for n in compute_topological_order(g):
        k = 1 + max((lvl[id(prod[i])] for i in n.inputs if i in prod), default=-1)
        lvl[id(n)] = k
        while len(levels) <= k:
            levels.append([])
        levels[k].append(n)
    return SchedulePlan(levels)


def analyze_parallelism(g: GraphIr) -> dict:
    s = generate_schedule(g)
    return {"depth": s.depth, "max_parallelism": s.max_parallelism,
            "mean_parallelism": (len(g.nodes) / s.depth) if s.depth else 0.0}


def max_parallelism(g: GraphIr) -> int:
    return generate_schedule(g).max_parallelism


def analyze_fusion_candidates(g: GraphIr) -> list[list[str]]:
    """Op names of each fusible group (elementwise chains after a producer) from the fusion planner."""
    by_id = {n.id: n for n in g.nodes}
    return [[by_id[i].op for i in grp] for grp in plan_fusion(g).groups]


def analyze_cycles(g: GraphIr) -> bool:
    try:
        compute_topological_order(g)
        return False
    except GraphError:
        return True


def _const_value(g: GraphIr, vid: int):
    v = g.values[vid]
    return None if v.constant is None else v.constant


def rewrite_algebraic(g: GraphIr) -> int:
    """Replace x * 1, 1 * x, x + 0, 0 + x, x - 0, x / 1 and identity nodes by x. Returns the count."""
    from .graph import _rename
    n_rw = 0
    for n in list(g.nodes):
        keep = None
        if n.op == "identity":
            keep = n.inputs[0]
        elif n.op in ("mul", "add", "sub", "div") and len(n.inputs) == 2:
            a, b = n.inputs
            ca, cb = _const_value(g, a), _const_value(g, b)
            neutral = 1.0 if n.op in ("mul", "div") else 0.0

            def is_neutral(c):
                return c is not None and c.numel() > 0 and bool((c == neutral).all())
            out_shape = g.values[n.outputs[0]].shape
            if is_neutral(cb) and g.values[a].shape == out_shape:
                keep = a
            elif n.op in ("mul", "add") and is_neutral(ca) and g.values[b].shape == out_shape:
                keep = b
        if keep is not None:
            old = n.outputs[0]
            if old in g.outputs:
                continue  # the output value keeps its producer
            g.nodes.remove(n)
            _rename(g, old, keep)
            n_rw += 1
    return n_rw


def clone_subgraph(g: GraphIr, output_vids) -> GraphIr:
    """A copy holding only what the given outputs depend on."""
    c = g.clone()
    c.outputs = list(output_vids)
    from .graph import eliminate_dead_code
    eliminate_dead_code(c)
    return c


@dataclass
class GraphProfile:
    per_node_ms: list = field(default_factory=list)  # (op, name, ms)

    @property
    def total_ms(self) -> float:
        return sum(t for _, _, t in self.per_node_ms)

    def top(self, k: int = 5):
        return sorted(self.per_node_ms, key=lambda r: -r[2])[:k]


def profile_graph(g: GraphIr, inputs, iters: int = 3) -> GraphProfile:
    """Per-node time (CUDA events on GPU inputs, wall clock on CPU), averaged over ``iters`` runs."""
    dev = inputs[0].device
    env = dict(zip(g.inputs, inputs))
    for vid, v in g.values.items():
        if v.constant is not None:
            env[vid] = v.constant.to(dev)
    acc = [0.0] * len(g.nodes)
    for _ in range(iters):
        for j, n in enumerate(g.nodes):
            xs = [env[i] for i in n.inputs]
            if dev.type == "cuda":
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                env[n.outputs[0]] = run_op(n.op, xs, n.attrs)
                e.record()
                e.synchronize()
                acc[j] += s.elapsed_time(e)
            else:
                t0 = time.perf_counter()
                env[n.outputs[0]] = run_op(n.op, xs, n.attrs)
                acc[j] += (time.perf_counter() - t0) * 1e3
    return GraphProfile([(n.op, g.values[n.outputs[0]].name, acc[j] / iters) for j, n in enumerate(g.nodes)])


def total_output_memory_bytes(g: GraphIr, elem_bytes: int = 4) -> int:
    tot = 0
    for n in g.nodes:
        shp = g.values[n.outputs[0]].shape
        if shp:
            k = 1
            for d in shp:
                k *= int(d)
            tot += k * elem_bytes
    return tot


def arithmetic_intensity(g: GraphIr, elem_bytes: int = 4) -> float:
    """Estimated FLOPs per byte of node outputs written (a lower bound on traffic)."""
    b = total_output_memory_bytes(g, elem_bytes)
    return estimate_flops(g) / b if b else 0.0


def format_graph_summary(g: GraphIr) -> str:
    ops: dict[str, int] = {}
    for n in g.nodes:
        ops[n.op] = ops.get(n.op, 0) + 1
    par = analyze_parallelism(g)
    lines = [f"graph {g.name}: {len(g.nodes)} nodes, {len(g.inputs)} inputs, {len(g.outputs)} outputs, "
             f"depth {par['depth']}, max parallelism {par['max_parallelism']}"]
    lines += [f"  {op}: {k}" for op, k in sorted(ops.items(), key=lambda kv: (-kv[1], kv[0]))]
    return "\n".join(lines)


def export_text(g: GraphIr) -> str:
    """One line per node: %out = op(%in, ...) {attrs}."""
    out = [f"graph {g.name}(" + ", ".join(f"%{i}" for i in g.inputs) + ")"]
    for n in g.nodes:
        attrs = " {" + ", ".join(f"{k}={v}" for k, v in sorted(n.attrs.items())) + "}" if n.attrs else ""
        out.append(f"  %{n.outputs[0]} = {n.op}(" + ", ".join(f"%{i}" for i in n.inputs) + f"){attrs}")
    out.append("  return " + ", ".join(f"%{o}" for o in g.outputs))
    return "\n".join(out)


def run_graph(g: GraphIr, inputs) -> list:
    return GraphInterpreter().run(g, list(inputs))


class ExecutionEngine:
    """Runs a graph repeatedly. On CUDA inputs the first call after ``prepare`` captures the node
    sequence into one CUDA graph over static input buffers; later calls copy the new inputs in and
    replay it (one launch for the whole graph). On the CPU it interprets."""

    def __init__(self, g: GraphIr, use_cuda_graph: bool = True):
        self.g, self.use_cuda_graph = g, use_cuda_graph
        self._graph = None
        self._static_in = None
        self._static_out = None

    def _capture(self, inputs):
        dev = inputs[0].device
        for v in self.g.values.values():  # constants live on the device, so the capture copies nothing from the host
            if v.constant is not None and v.constant.device != dev:
                v.constant = v.constant.to(dev)
        self._static_in = [x.clone() for x in inputs]
        interp = GraphInterpreter()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            interp.run(self.g, self._static_in)  # warm-up allocations and lazy kernel loads outside the capture
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._static_out = interp.run(self.g, self._static_in)
        self._graph = graph

    def run(self, inputs) -> list:
        inputs = list(inputs)
        if not (self.use_cuda_graph and inputs and inputs[0].is_cuda):
            return GraphInterpreter().run(self.g, inputs)
        if self._graph is None or any(a.shape != b.shape for a, b in zip(self._static_in, inputs)):
            self._capture(inputs)
        for s, x in zip(self._static_in, inputs):
            s.copy_(x)
        self._graph.replay()
        return [o.clone() for o in self._static_out]
