"""Graph IR, optimisation passes, interpreter, planners and exporters.

Reference: crates/brain-graph (``GraphIr`` with values and nodes, ir/mod.rs:19-120; verification
ir/verify.rs; shape inference ir/shape_infer.rs; passes const-fold / DCE / CSE / layout / fusion plan /
in-place plan, passes/*.rs, driven by ``PassManager`` passes/mod.rs:33-60 and ``optimize(level)``
optimize.rs:15-60; ``GraphInterpreter`` interp.rs:14-60; DOT and JSON export dot.rs, json.rs;
``diff_graphs`` diff.rs:10-40) and crates/brain-compile (FLOP estimate, memory plan and schedule,
plan.rs; the JIT cache jit.rs:11-40).

Design: a small SSA IR whose op set is the framework's own fused operations. The interpreter runs each
node with torch on the inputs' device, and ``matmul`` / ``linear`` nodes on CUDA bf16 go through the
framework's tcgen05 GEMM (``ops.gemm``). The fusion planner groups a GEMM with the elementwise chain
that follows it (bias, residual add, activation) where a single GEMM epilogue of this framework can
absorb it, and the memory planner assigns values to reusable buffers by liveness (greedy best fit).
``from_fx`` captures a ``torch.nn.Module`` through ``torch.fx`` into this IR.
"""
from __future__ import annotations

import copy
import json
import math
from dataclasses import dataclass, field

import torch

# op -> (arity or None for variadic, elementwise?)
ELEMENTWISE_UNARY = {"relu", "gelu", "silu", "tanh", "sigmoid", "exp", "log", "neg", "sqrt", "rsqrt", "abs"}
ELEMENTWISE_BINARY = {"add", "sub", "mul", "div", "maximum", "minimum", "pow"}
OPS = ELEMENTWISE_UNARY | ELEMENTWISE_BINARY | {
    "matmul", "linear", "transpose", "reshape", "softmax", "log_softmax", "sum", "mean", "layer_norm",
    "rms_norm", "swiglu", "concat", "identity", "constant_scale"}


class GraphError(RuntimeError):
    pass


@dataclass
class GraphValue:
    id: int
    name: str
    shape: tuple | None = None
    dtype: str = "float32"
    constant: torch.Tensor | None = None


@dataclass
class GraphNode:
    id: int
    op: str
    inputs: list[int]
    outputs: list[int]
    attrs: dict = field(default_factory=dict)


class GraphIr:
    def __init__(self, name: str = "graph"):
        self.name = name
        self.values: dict[int, GraphValue] = {}
        self.nodes: list[GraphNode] = []
        self.inputs: list[int] = []
        self.outputs: list[int] = []
        self._next = 0

    # ---- building
    def _id(self) -> int:
        self._next += 1
        return self._next - 1

    def add_value(self, name: str, shape=None, dtype: str = "float32") -> int:
        i = self._id()
        self.values[i] = GraphValue(i, name, tuple(shape) if shape is not None else None, dtype)
        return i

    def add_input(self, name: str, shape=None, dtype: str = "float32") -> int:
        i = self.add_value(name, shape, dtype)
        self.inputs.append(i)
        return i

    def set_constant(self, vid: int, data) -> None:
        t = torch.as_tensor(data)
        v = self.values[vid]
        v.constant, v.shape, v.dtype = t, tuple(t.shape), str(t.dtype).replace("torch.", "")

    def constant(self, name: str, data) -> int:
        i = self.add_value(name)
        self.set_constant(i, data)
        return i

    def add_node(self, op: str, inputs, attrs=None, name: str | None = None, num_outputs: int = 1):
        if op not in OPS:
            raise GraphError(f"unknown op {op!r}")
        outs = [self.add_value(name or f"{op}_{len(self.nodes)}" + (f".{k}" if num_outputs > 1 else ""))
                for k in range(num_outputs)]
        self.nodes.append(GraphNode(self._id(), op, list(inputs), outs, dict(attrs or {})))
        return outs[0] if num_outputs == 1 else outs

    def mark_output(self, *vids) -> None:
        self.outputs.extend(vids)

    def get_node(self, nid):
        return next((n for n in self.nodes if n.id == nid), None)

    def get_value(self, vid):
        return self.values.get(vid)

    def num_nodes(self) -> int:
        return len(self.nodes)

    def num_values(self) -> int:
        return len(self.values)

    def producers(self) -> dict[int, GraphNode]:
        return {o: n for n in self.nodes for o in n.outputs}

    def consumers(self) -> dict[int, list[GraphNode]]:
        out: dict[int, list[GraphNode]] = {}
        for n in self.nodes:
            for i in n.inputs:
                out.setdefault(i, []).append(n)
        return out

    def clone(self) -> "GraphIr":
        return copy.deepcopy(self)


# ------------------------------------------------------------------ op semantics
def _act(name, x):
    return {"relu": torch.relu, "gelu": lambda t: torch.nn.functional.gelu(t, approximate="tanh"),
            "silu": torch.nn.functional.silu, "tanh": torch.tanh, "sigmoid": torch.sigmoid, "exp": torch.exp,
            "log": torch.log, "neg": torch.neg, "sqrt": torch.sqrt, "rsqrt": torch.rsqrt, "abs": torch.abs}[name](x)


def _matmul(a, b):
    if a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16 and a.dim() >= 2 and b.dim() == 2:
        from . import ops
        lead = a.shape[:-1]
        return ops.gemm(a.reshape(-1, a.shape[-1]), b).reshape(*lead, b.shape[-1])
    return torch.matmul(a, b)


def run_op(op: str, xs: list, attrs: dict):
    if op == "gelu" and attrs.get("approximate", "tanh") != "tanh":
        return torch.nn.functional.gelu(xs[0], approximate=attrs["approximate"])
    if op in ELEMENTWISE_UNARY:
        return _act(op, xs[0])
    if op in ELEMENTWISE_BINARY:
        f = {"add": torch.add, "sub": torch.sub, "mul": torch.mul, "div": torch.div, "maximum": torch.maximum,
             "minimum": torch.minimum, "pow": torch.pow}[op]
        return f(xs[0], xs[1])
    if op == "matmul":
        return _matmul(xs[0], xs[1])
    if op == "linear":  # x W^T (+ b)
        b = xs[2] if len(xs) > 2 else None
        if xs[0].is_cuda and xs[0].dtype == torch.bfloat16:
            from . import ops
            return ops.linear(xs[0], xs[1], b)
        return torch.nn.functional.linear(xs[0], xs[1], b)
    if op == "transpose":
        return xs[0].transpose(attrs.get("dim0", -2), attrs.get("dim1", -1))
    if op == "reshape":
        return xs[0].reshape(attrs["shape"])
    if op == "softmax":
        return torch.softmax(xs[0], attrs.get("dim", -1))
    if op == "log_softmax":
        return torch.log_softmax(xs[0], attrs.get("dim", -1))
    if op == "sum":
        return xs[0].sum(attrs.get("dim"), keepdim=attrs.get("keepdim", False)) if "dim" in attrs else xs[0].sum()
    if op == "mean":
        return xs[0].mean(attrs.get("dim"), keepdim=attrs.get("keepdim", False)) if "dim" in attrs else xs[0].mean()
    if op == "layer_norm":
        return torch.nn.functional.layer_norm(xs[0], xs[0].shape[-1:], xs[1] if len(xs) > 1 else None,
                                              xs[2] if len(xs) > 2 else None, attrs.get("eps", 1e-5))
    if op == "rms_norm":
        x = xs[0]
        y = x * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + attrs.get("eps", 1e-6)).to(x.dtype)
        return y * xs[1] if len(xs) > 1 else y
    if op == "swiglu":
        g, u = xs[0].chunk(2, -1) if len(xs) == 1 else (xs[0], xs[1])
        return torch.nn.functional.silu(g) * u
    if op == "concat":
        return torch.cat(xs, attrs.get("dim", -1))
    if op == "identity":
        return xs[0]
    if op == "constant_scale":
        return xs[0] * attrs["scale"]
    raise GraphError(f"no implementation for {op}")


def infer_shapes(g: GraphIr, input_shapes: dict | None = None) -> None:
    """Propagates shapes by running every node on meta tensors."""
    env = {}
    for vid in g.inputs:
        shp = (input_shapes or {}).get(vid, g.values[vid].shape)
        if shp is None:
            raise GraphError(f"input {g.values[vid].name} has no shape")
        env[vid] = torch.empty(shp, device="meta")
    for vid, v in g.values.items():
        if v.constant is not None:
            env[vid] = torch.empty(v.shape, device="meta", dtype=v.constant.dtype)
    for n in g.nodes:
        xs = [env[i] for i in n.inputs]
        if n.op in ("matmul", "linear"):
            y = torch.matmul(xs[0], xs[1] if n.op == "matmul" else xs[1].t())
        elif n.op in ("layer_norm", "rms_norm"):
            y = torch.empty_like(xs[0])
        else:
            y = run_op(n.op, xs, n.attrs)
        env[n.outputs[0]] = y
        g.values[n.outputs[0]].shape = tuple(y.shape)


def verify(g: GraphIr) -> list[str]:
    """Every input defined before use, one producer per value, outputs defined, known ops."""
    errs, defined = [], set(g.inputs) | {v for v, x in g.values.items() if x.constant is not None}
    produced = set()
    for n in g.nodes:
        if n.op not in OPS:
            errs.append(f"node {n.id}: unknown op {n.op}")
        for i in n.inputs:
            if i not in defined:
                errs.append(f"node {n.id} ({n.op}) uses undefined value {i}")
        for o in n.outputs:
            if o in produced or o in g.inputs:
                errs.append(f"value {o} has more than one producer")
            produced.add(o)
            defined.add(o)
    for o in g.outputs:
        if o not in defined:
            errs.append(f"graph output {o} is never defined")
    return errs


# ------------------------------------------------------------------ passes
def fold_constants(g: GraphIr) -> bool:
    changed = False
    keep = []
    for n in g.nodes:
        if n.inputs and all(g.values[i].constant is not None for i in n.inputs) and len(n.outputs) == 1:
            g.set_constant(n.outputs[0], run_op(n.op, [g.values[i].constant for i in n.inputs], n.attrs))
            changed = True
        else:
            keep.append(n)
    g.nodes = keep
    return changed


def eliminate_dead_code(g: GraphIr) -> bool:
    live = set(g.outputs)
    keep = []
    for n in reversed(g.nodes):
        if any(o in live for o in n.outputs):
            keep.append(n)
            live.update(n.inputs)
    keep.reverse()
    changed = len(keep) != len(g.nodes)
    g.nodes = keep
    used = live | set(g.inputs)
    for vid in [v for v in g.values if v not in used and not any(v in n.outputs for n in keep)]:
        del g.values[vid]
    return changed


def _rename(g: GraphIr, old: int, new: int) -> None:
    for n in g.nodes:
        n.inputs = [new if i == old else i for i in n.inputs]
    g.outputs = [new if o == old else o for o in g.outputs]


def eliminate_cse(g: GraphIr) -> bool:
    seen, changed, keep = {}, False, []
    for n in g.nodes:
        key = (n.op, tuple(n.inputs), json.dumps(n.attrs, sort_keys=True, default=str))
        if key in seen and len(n.outputs) == 1:
            _rename(g, n.outputs[0], seen[key])
            changed = True
            continue
        seen[key] = n.outputs[0]
        keep.append(n)
    g.nodes = keep
    return changed


def eliminate_layout_transforms(g: GraphIr) -> bool:
    """transpose(transpose(x)) over the same dims -> x; reshape of a reshape -> one reshape;
    identity -> its input."""
    prod = g.producers()
    changed = False
    for n in g.nodes:
        src = prod.get(n.inputs[0]) if n.inputs else None
        if n.op == "identity":
            _rename(g, n.outputs[0], n.inputs[0])
            changed = True
        elif n.op == "transpose" and src is not None and src.op == "transpose":
            d = lambda a: tuple(sorted((a.get("dim0", -2), a.get("dim1", -1))))  # noqa: E731
            if d(n.attrs) == d(src.attrs):
                _rename(g, n.outputs[0], src.inputs[0])
                changed = True
        elif n.op == "reshape" and src is not None and src.op == "reshape":
            n.inputs = [src.inputs[0]]
            changed = True
    if changed:
        eliminate_dead_code(g)
    return changed


@dataclass
class FusionPlan:
    groups: list[list[int]]  # node ids; the first is the anchor (GEMM or norm)

    def num_fused(self) -> int:
        return sum(len(x) - 1 for x in self.groups)


def plan_fusion(g: GraphIr) -> FusionPlan:
    """A GEMM (matmul / linear) followed by a single-consumer chain of bias add, residual add and one
    activation is one group: the framework's GEMM epilogue applies bias, residual and activation on the
    accumulators. A norm followed by a linear is a group too (the norm is recomputed in the fused
    layer's backward)."""
    cons = g.consumers()
    groups, taken = [], set()
    for n in g.nodes:
        if n.id in taken:
            continue
        if n.op in ("matmul", "linear"):
            grp, cur, acts = [n.id], n, 0
            while True:
                nxt = cons.get(cur.outputs[0], [])
                if len(nxt) != 1 or cur.outputs[0] in g.outputs:
                    break
                m = nxt[0]
                if m.op == "add" or (m.op in ELEMENTWISE_UNARY and acts == 0 and m.op in ("relu", "gelu", "silu")):
                    acts += m.op != "add"
                    grp.append(m.id)
                    cur = m
                else:
                    break
            if len(grp) > 1:
                groups.append(grp)
                taken.update(grp)
        elif n.op in ("rms_norm", "layer_norm"):
            nxt = cons.get(n.outputs[0], [])
            if len(nxt) == 1 and nxt[0].op == "linear" and nxt[0].id not in taken:
                groups.append([n.id, nxt[0].id])
                taken.update((n.id, nxt[0].id))
    return FusionPlan(groups)


@dataclass
class InplacePlan:
    inplace: dict[int, int]  # node id -> input value whose storage it may overwrite


def plan_inplace_operations(g: GraphIr) -> InplacePlan:
    """An elementwise node may write into an input whose last use it is (and which is not a graph
    input, output or constant)."""
    last_use = {}
    for idx, n in enumerate(g.nodes):
        for i in n.inputs:
            last_use[i] = idx
    plan = {}
    for idx, n in enumerate(g.nodes):
        if n.op not in ELEMENTWISE_UNARY | ELEMENTWISE_BINARY:
            continue
        for i in n.inputs:
            v = g.values[i]
            if last_use.get(i) == idx and i not in g.inputs and i not in g.outputs and v.constant is None:
                plan[n.id] = i
                break
    return InplacePlan(plan)


class PassManager:
    def __init__(self):
        self.passes = []

    def add_pass(self, fn) -> None:
        self.passes.append(fn)

    def run(self, g: GraphIr, max_iterations: int = 10) -> int:
        it = 0
        for it in range(1, max_iterations + 1):
            if not any([p(g) for p in self.passes]):
                break
        return it


@dataclass
class OptimizeReport:
    nodes_before: int
    nodes_after: int
    iterations: int
    fusion: FusionPlan | None = None


def optimize(g: GraphIr, level: int = 2) -> OptimizeReport:
    """Level 0: nothing. 1: const-fold + DCE. 2: + CSE + layout cleanup + fusion plan."""
    before = g.num_nodes()
    if level <= 0:
        return OptimizeReport(before, before, 0)
    pm = PassManager()
    pm.add_pass(fold_constants)
    if level >= 2:
        pm.add_pass(eliminate_cse)
        pm.add_pass(eliminate_layout_transforms)
    pm.add_pass(eliminate_dead_code)
    it = pm.run(g)
    return OptimizeReport(before, g.num_nodes(), it, plan_fusion(g) if level >= 2 else None)


# ------------------------------------------------------------------ execution
class GraphInterpreter:
    def run(self, g: GraphIr, inputs: list[torch.Tensor]) -> list[torch.Tensor]:
        if len(inputs) != len(g.inputs):
            raise GraphError(f"expected {len(g.inputs)} inputs, got {len(inputs)}")
        dev = inputs[0].device if inputs else None
        env = dict(zip(g.inputs, inputs))
        for vid, v in g.values.items():
            if v.constant is not None:
                env[vid] = v.constant.to(dev) if dev is not None else v.constant
        for n in g.nodes:
            env[n.outputs[0]] = run_op(n.op, [env[i] for i in n.inputs], n.attrs)
        return [env[o] for o in g.outputs]


def estimate_flops(g: GraphIr) -> int:
    """2 M N K per GEMM plus one FLOP per output element of every other node (shapes must be known)."""
    tot = 0
    for n in g.nodes:
        out = g.values[n.outputs[0]].shape
        numel = math.prod(out) if out else 1
        if n.op in ("matmul", "linear"):
            k = g.values[n.inputs[0]].shape[-1]
            tot += 2 * numel * k
        else:
            tot += numel
    return tot


@dataclass
class MemoryPlan:
    assignment: dict[int, int]  # value id -> buffer index
    buffer_bytes: list[int]

    def total_bytes(self) -> int:
        return sum(self.buffer_bytes)


def plan_memory(g: GraphIr, elem_bytes: int = 4) -> MemoryPlan:
    """Liveness-based reuse of intermediate buffers (greedy best fit in schedule order)."""
    last = {}
    for idx, n in enumerate(g.nodes):
        for i in n.inputs:
            last[i] = idx
    for o in g.outputs:
        last[o] = len(g.nodes)
    free: list[int] = []
    sizes: list[int] = []
    assign = {}
    for idx, n in enumerate(g.nodes):
        o = n.outputs[0]
        need = math.prod(g.values[o].shape or (1,)) * elem_bytes
        fits = sorted((sizes[b], b) for b in free if sizes[b] >= need)
        if fits:
            b = fits[0][1]
            free.remove(b)
        else:
            b = len(sizes)
            sizes.append(need)
        assign[o] = b
        for i in set(n.inputs):
            if i in assign and last.get(i) == idx:
                free.append(assign[i])
    return MemoryPlan(assign, sizes)


class JitCache:
    """Caches optimised graphs per (graph signature, options) so repeated compiles are free."""

    def __init__(self):
        self._cache = {}
        self.hits = self.misses = 0

    def get_or_compile(self, g: GraphIr, level: int = 2) -> GraphIr:
        key = (to_json(g), level)
        if key in self._cache:
            self.hits += 1
            return self._cache[key]
        self.misses += 1
        h = g.clone()
        optimize(h, level)
        self._cache[key] = h
        return h


# ------------------------------------------------------------------ export / diff / capture
def to_dot(g: GraphIr) -> str:
    lines = [f'digraph "{g.name}" {{', "  rankdir=LR;"]
    for vid in g.inputs:
        lines.append(f'  v{vid} [shape=ellipse,label="{g.values[vid].name}"];')
    for n in g.nodes:
        lines.append(f'  n{n.id} [shape=box,label="{n.op}"];')
        for i in n.inputs:
            src = next((m for m in g.nodes if i in m.outputs), None)
            lines.append(f"  {'n%d' % src.id if src else 'v%d' % i} -> n{n.id};")
    lines.append("}")
    return "\n".join(lines)


def to_json(g: GraphIr) -> str:
    return json.dumps({
        "name": g.name, "inputs": g.inputs, "outputs": g.outputs,
        "values": [{"id": v.id, "name": v.name, "shape": v.shape, "dtype": v.dtype,
                    "constant": v.constant.tolist() if v.constant is not None else None} for v in g.values.values()],
        "nodes": [{"id": n.id, "op": n.op, "inputs": n.inputs, "outputs": n.outputs, "attrs": n.attrs}
                  for n in g.nodes]}, sort_keys=True)


def from_json(s: str) -> GraphIr:
    d = json.loads(s)
    g = GraphIr(d["name"])
    for v in d["values"]:
        g.values[v["id"]] = GraphValue(v["id"], v["name"], tuple(v["shape"]) if v["shape"] is not None else None,
                                       v["dtype"], torch.tensor(v["constant"]) if v["constant"] is not None else None)
    g.nodes = [GraphNode(n["id"], n["op"], n["inputs"], n["outputs"], n["attrs"]) for n in d["nodes"]]
    g.inputs, g.outputs = d["inputs"], d["outputs"]
    g._next = 1 + max([*g.values, *(n.id for n in g.nodes), -1])
    return g


@dataclass
class GraphDiff:
    added_ops: dict
    removed_ops: dict
    nodes_a: int
    nodes_b: int

    def is_empty(self) -> bool:
        return not self.added_ops and not self.removed_ops


def diff_graphs(a: GraphIr, b: GraphIr) -> GraphDiff:
    from collections import Counter

    ca, cb = Counter(n.op for n in a.nodes), Counter(n.op for n in b.nodes)
    return GraphDiff(dict(cb - ca), dict(ca - cb), a.num_nodes(), b.num_nodes())


_FX_FUNCS = {torch.relu: "relu", torch.tanh: "tanh", torch.sigmoid: "sigmoid", torch.exp: "exp",
             torch.matmul: "matmul", torch.add: "add", torch.mul: "mul", torch.sub: "sub",
             torch.nn.functional.relu: "relu", torch.nn.functional.silu: "silu", torch.nn.functional.gelu: "gelu"}


def from_fx(module: torch.nn.Module, *example_inputs) -> GraphIr:
    """Captures ``module`` with ``torch.fx.symbolic_trace``: Linear / activation modules, arithmetic
    operators and the functions above become IR nodes; parameters become constants. Shapes come from
    the example inputs."""
    import operator

    import torch.fx as fx

    gm = fx.symbolic_trace(module)
    g = GraphIr(type(module).__name__)
    env = {}
    mods = dict(gm.named_modules())
    binops = {operator.add: "add", operator.mul: "mul", operator.sub: "sub", operator.truediv: "div",
              operator.matmul: "matmul"}
    ex = iter(example_inputs)
    for node in gm.graph.nodes:
        if node.op == "placeholder":
            t = next(ex)
            env[node.name] = g.add_input(node.name, tuple(t.shape), str(t.dtype).replace("torch.", ""))
        elif node.op == "get_attr":
            env[node.name] = g.constant(node.target, getattr(gm, node.target).detach())
        elif node.op == "call_module":
            m = mods[node.target]
            x = env[node.args[0].name]
            if isinstance(m, torch.nn.Linear) or type(m).__name__ == "Linear":
                w = g.constant(f"{node.target}.weight", m.weight.detach())
                ins = [x, w] + ([g.constant(f"{node.target}.bias", m.bias.detach())] if m.bias is not None else [])
                env[node.name] = g.add_node("linear", ins, name=node.name)
            else:
                op = {torch.nn.ReLU: "relu", torch.nn.Tanh: "tanh", torch.nn.Sigmoid: "sigmoid", torch.nn.SiLU: "silu",
                      torch.nn.GELU: "gelu", torch.nn.Identity: "identity"}.get(type(m))
                if op is None:
                    raise GraphError(f"unsupported module {type(m).__name__}")
                attrs = {"approximate": m.approximate} if op == "gelu" else None
                env[node.name] = g.add_node(op, [x], attrs, name=node.name)
        elif node.op in ("call_function", "call_method"):
            tgt = node.target
            op = binops.get(tgt) or _FX_FUNCS.get(tgt) or (tgt if isinstance(tgt, str) and tgt in OPS else None)
            if op is None:
                raise GraphError(f"unsupported function {tgt}")
            ins = []
            for a in node.args:
                if isinstance(a, fx.Node):
                    ins.append(env[a.name])
                else:
                    ins.append(g.constant(f"c{len(g.values)}", torch.tensor(float(a))))
            attrs = {"approximate": node.kwargs.get("approximate", "none")} if op == "gelu" else None
            env[node.name] = g.add_node(op, ins, attrs, name=node.name)
        elif node.op == "output":
            outs = node.args[0] if isinstance(node.args[0], (tuple, list)) else (node.args[0],)
            g.mark_output(*[env[o.name] for o in outs])
    infer_shapes(g)
    return g
