"""Graph utilities over the recorded backward graph: ``topological_sort`` (iterative post-order DFS with
cycle detection), ``compute_dag_levels`` (longest-path levels from the leaves), ``values_close``,
``TapeBuilder`` and ``RecomputeGraph``.

Reference: crates/brain-autograd/src/backward/topo.rs:22-98, value.rs:634-645, tape/builder.rs:9-30,
checkpoint/offload.rs:10-33.

A ``Value`` here wraps a torch tensor whose backward graph is torch's (``grad_fn`` nodes linked by
``next_functions``; a leaf that requires grad appears as an ``AccumulateGrad`` node). The traversal
walks that graph, so it covers every op the framework's kernels register with autograd, not only the
ones the ``Value`` wrapper records on a tape.
"""
from __future__ import annotations

import torch

from .tape import OpRecord, Tape
from .value import Value


def _root(x):
    t = x.tensor if isinstance(x, Value) else x
    if isinstance(t, torch.Tensor):
        return t.grad_fn
    return t  # already a graph node


def _parents(node) -> list:
    return [p for p, _ in getattr(node, "next_functions", ()) if p is not None]


def topological_sort(root) -> list:
    """Graph nodes reachable from ``root`` (a Value, a tensor or a grad_fn node), inputs before the nodes
    that consume them, the root last. Iterative, so graphs thousands of ops deep do not exhaust the
    Python stack. Raises ValueError on a cycle."""
    node = _root(root)
    if node is None:
        return []
    order, done, active = [], set(), set()
    stack = [(node, False)]
    while stack:
        n, finalize = stack.pop()
        k = id(n)
        if finalize:
            active.discard(k)
            done.add(k)
            order.append(n)
            continue
        if k in active:
            raise ValueError(f"cycle detected in computation graph at node {type(n).__name__}")
        if k in done:
            continue
        active.add(k)
        stack.append((n, True))
        for p in _parents(n):
            if id(p) not in done:
                stack.append((p, False))
    return order


def compute_dag_levels(ordered_nodes: list) -> list[list]:
    """Bucket nodes (in topological order) by longest dependency chain from a leaf: level 0 holds the
    leaves, level k = 1 + the maximum level of the node's inputs. Nodes in one level are independent."""
    level: dict[int, int] = {}
    buckets: list[list] = []
    for n in ordered_nodes:
        ps = _parents(n)
        lv = 1 + max(level.get(id(p), 0) for p in ps) if ps else 0
        level[id(n)] = lv
        while len(buckets) <= lv:
            buckets.append([])
        buckets[lv].append(n)
    return buckets


def values_close(a, b, tol: float) -> bool:
    """Same shape and every element within ``tol`` (absolute)."""
    ta = a.tensor if isinstance(a, Value) else torch.as_tensor(a)
    tb = b.tensor if isinstance(b, Value) else torch.as_tensor(b)
    if ta.shape != tb.shape:
        return False
    return bool(((ta.detach().double() - tb.detach().double()).abs() <= tol).all())


class TapeBuilder:
    """Fluent construction of a tape: ``TapeBuilder().add_op(rec).add_op(rec2).build()``."""

    def __init__(self):
        self._tape = Tape()

    def add_op(self, op: OpRecord) -> "TapeBuilder":
        self._tape.records.append(op)
        return self

    def build(self) -> Tape:
        return self._tape


class RecomputeGraph:
    """A deferred recomputation: the saved inputs of one op and the function that recomputes its output
    during backward (activation checkpointing keeps this instead of the output)."""

    def __init__(self, inputs: list, op_name: str, fn=None):
        self.inputs, self._op, self._fn = list(inputs), op_name, fn

    def input_count(self) -> int:
        return len(self.inputs)

    def op_name(self) -> str:
        return self._op

    def recompute(self):
        if self._fn is None:
            raise RuntimeError(f"no recompute function stored for {self._op!r}")
        return self._fn(*self.inputs)
