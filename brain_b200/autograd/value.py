"""``Value``: the reference's dynamic-graph autograd node, backed by torch autograd.

Reference: crates/brain-autograd/src/value.rs (``Value::new``, op methods at :300-560 including
``linear`` :514 and ``embedding`` :529, ``backward`` :292, ``accumulate_grad`` summing to shape
for broadcasts :266) and the GradFn VJPs (grad_fns/mod.rs:20-101). Here each Value holds a
``torch.Tensor``; the graph, topological sort and VJPs are PyTorch's engine, the heavy ops
(``linear``, ``embedding``, ``softmax_cross_entropy``, attention) route to the sm_100a kernels on
CUDA. Broadcasting gradients are reduced to the operand's shape by torch, which is the
reference's ``sum_to_shape``. Deep chains do not recurse on drop (the reference makes ``Drop``
iterative for 100k-deep chains; torch's graph teardown is iterative as well).
"""
from __future__ import annotations

import itertools

import torch

from .. import ops
from . import tape as _tape

_ids = itertools.count()


def _t(x) -> torch.Tensor:
    if isinstance(x, Value):
        return x.tensor
    if isinstance(x, torch.Tensor):
        return x
    return torch.as_tensor(x)


class Value:
    __slots__ = ("tensor", "id", "name", "op")

    def __init__(self, data, requires_grad: bool = False, name: str | None = None, _op: str = "leaf"):
        t = data.tensor if isinstance(data, Value) else torch.as_tensor(data)
        if requires_grad and not t.requires_grad:
            if not t.is_leaf:
                t = t.detach()
            if not t.is_floating_point():
                t = t.float()
            t.requires_grad_(True)
        self.tensor = t
        self.id = next(_ids)
        self.name = name
        self.op = _op

    # ------------------------------------------------------------------ construction / access
    @staticmethod
    def new(tensor, requires_grad: bool = False) -> "Value":
        return Value(tensor, requires_grad)

    @staticmethod
    def parameter(tensor) -> "Value":
        return Value(tensor, True)

    @staticmethod
    def _wrap(t: torch.Tensor, op: str, *parents) -> "Value":
        v = Value(t, _op=op)
        _tape.record(op, [p.id for p in parents if isinstance(p, Value)], v.id, tuple(t.shape))
        return v

    def data(self) -> torch.Tensor:
        return self.tensor.detach()

    def grad(self) -> torch.Tensor | None:
        g = self.tensor.grad
        return None if g is None else g.detach()

    @property
    def requires_grad(self) -> bool:
        return self.tensor.requires_grad

    @property
    def is_leaf(self) -> bool:
        return self.tensor.is_leaf

    @property
    def shape(self):
        return tuple(self.tensor.shape)

    def item(self) -> float:
        return float(self.tensor.item())

    def zero_grad(self) -> None:
        self.tensor.grad = None

    def detach(self) -> "Value":
        return Value(self.tensor.detach())

    def backward(self, grad: torch.Tensor | None = None, retain_graph: bool = False) -> None:
        """Seed with ones (the reference's ``backward_from``) and accumulate into leaves."""
        g = torch.ones_like(self.tensor) if grad is None else _t(grad).to(self.tensor)
        self.tensor.backward(g, retain_graph=retain_graph)

    def __repr__(self):
        return f"Value(id={self.id}, op={self.op}, shape={self.shape}, requires_grad={self.requires_grad})"

    # ------------------------------------------------------------------ binary ops
    def add(self, o):
        return Value._wrap(self.tensor + _t(o), "add", self, o)

    def sub(self, o):
        return Value._wrap(self.tensor - _t(o), "sub", self, o)

    def mul(self, o):
        return Value._wrap(self.tensor * _t(o), "mul", self, o)

    def div(self, o):
        return Value._wrap(self.tensor / _t(o), "div", self, o)

    def pow(self, e):
        return Value._wrap(self.tensor ** _t(e), "pow", self, e)

    def matmul(self, o):
        a, b = self.tensor, _t(o)
        if a.is_cuda and a.dim() == 2 and b.dim() == 2 and a.dtype == torch.bfloat16:
            out = ops.linear(a, b.t().contiguous())
        else:
            out = a @ b
        return Value._wrap(out, "matmul", self, o)

    def minimum(self, o):
        return Value._wrap(torch.minimum(self.tensor, _t(o)), "min_elem", self, o)

    def maximum(self, o):
        return Value._wrap(torch.maximum(self.tensor, _t(o)), "max_elem", self, o)

    __add__ = add
    __sub__ = sub
    __mul__ = mul
    __truediv__ = div
    __matmul__ = matmul
    __pow__ = pow

    def __radd__(self, o):
        return Value._wrap(_t(o) + self.tensor, "add", o, self)

    def __rsub__(self, o):
        return Value._wrap(_t(o) - self.tensor, "sub", o, self)

    def __rmul__(self, o):
        return Value._wrap(_t(o) * self.tensor, "mul", o, self)

    def __rtruediv__(self, o):
        return Value._wrap(_t(o) / self.tensor, "div", o, self)

    def __neg__(self):
        return self.neg()

    # ------------------------------------------------------------------ unary ops
    def _u(self, fn, name):
        return Value._wrap(fn(self.tensor), name, self)

    def neg(self):
        return self._u(torch.neg, "neg")

    def exp(self):
        return self._u(torch.exp, "exp")

    def log(self):
        return self._u(torch.log, "log")

    def sqrt(self):
        return self._u(torch.sqrt, "sqrt")

    def abs(self):
        return self._u(torch.abs, "abs")

    def sin(self):
        return self._u(torch.sin, "sin")

    def cos(self):
        return self._u(torch.cos, "cos")

    def tanh(self):
        return self._u(torch.tanh, "tanh")

    def sigmoid(self):
        return self._u(torch.sigmoid, "sigmoid")

    def relu(self):
        return self._u(torch.relu, "relu")

    def gelu(self):
        return self._u(ops.gelu, "gelu")

    def silu(self):
        return self._u(torch.nn.functional.silu, "silu")

    def sign(self):
        return self._u(torch.sign, "sign")

    def clamp(self, lo=None, hi=None):
        return Value._wrap(torch.clamp(self.tensor, lo, hi), "clamp", self)

    def softmax(self, dim: int = -1):
        t = self.tensor
        return Value._wrap(torch.softmax(t - t.amax(dim, keepdim=True).detach(), dim), "softmax", self)

    def log_softmax(self, dim: int = -1):
        return Value._wrap(torch.log_softmax(self.tensor, dim), "log_softmax", self)

    # ------------------------------------------------------------------ reductions / shape
    def sum(self, dim=None, keepdim=False):
        return Value._wrap(self.tensor.sum() if dim is None else self.tensor.sum(dim, keepdim), "sum", self)

    def mean(self, dim=None, keepdim=False):
        return Value._wrap(self.tensor.mean() if dim is None else self.tensor.mean(dim, keepdim), "mean", self)

    def max(self, dim=None):
        return Value._wrap(self.tensor.max() if dim is None else self.tensor.max(dim).values, "max", self)

    def reshape(self, *shape):
        return Value._wrap(self.tensor.reshape(*shape), "reshape", self)

    view = reshape

    def transpose(self, a=-2, b=-1):
        return Value._wrap(self.tensor.transpose(a, b), "transpose", self)

    def permute(self, *dims):
        return Value._wrap(self.tensor.permute(*dims), "permute", self)

    def index_select(self, dim, idx):
        return Value._wrap(self.tensor.index_select(dim, _t(idx)), "index_select", self)

    def where(self, cond, other):
        return Value._wrap(torch.where(_t(cond), self.tensor, _t(other)), "where", self, other)

    # ------------------------------------------------------------------ layers
    def linear(self, weight, bias=None):
        """x @ W^T + b (the reference's Value::linear)."""
        return Value._wrap(ops.linear(self.tensor, _t(weight), None if bias is None else _t(bias)), "linear",
                           self, weight, bias)

    def embedding(self, ids):
        """Rows of this [V, D] table gathered by ids (the reference's Value::embedding)."""
        return Value._wrap(ops.embedding(_t(ids), self.tensor), "embedding", self)

    def rms_norm(self, weight, eps=1e-6):
        return Value._wrap(ops.rms_norm(self.tensor, _t(weight), eps), "rms_norm", self, weight)

    def layer_norm(self, weight, bias=None, eps=1e-5):
        return Value._wrap(ops.layer_norm(self.tensor, _t(weight), None if bias is None else _t(bias), eps),
                           "layer_norm", self, weight, bias)

    def cross_entropy(self, targets, ignore_index=-100, label_smoothing=0.0):
        return Value._wrap(ops.cross_entropy(self.tensor, _t(targets), ignore_index, label_smoothing),
                           "cross_entropy", self)

    def conv2d(self, weight, bias=None, stride=1, padding=0):
        return Value._wrap(torch.nn.functional.conv2d(self.tensor, _t(weight), None if bias is None else _t(bias),
                                                      stride, padding), "conv2d", self, weight, bias)

    def max_pool2d(self, k, stride=None):
        return Value._wrap(torch.nn.functional.max_pool2d(self.tensor, k, stride), "max_pool2d", self)

    def adaptive_avg_pool2d(self, out_hw):
        return Value._wrap(torch.nn.functional.adaptive_avg_pool2d(self.tensor, out_hw), "adaptive_avg_pool2d", self)

    def adaptive_max_pool2d(self, out_hw):
        return Value._wrap(torch.nn.functional.adaptive_max_pool2d(self.tensor, out_hw), "adaptive_max_pool2d", self)

    def conv_transpose2d(self, weight, bias=None, stride=1, padding=0):
        w, b = _t(weight), (None if bias is None else _t(bias))
        return Value._wrap(torch.nn.functional.conv_transpose2d(self.tensor, w, b, stride, padding), "conv_transpose2d",
                           self, weight, bias)

    def where_cond(self, cond, other):
        """self where cond else other (the reference's ``where_cond``)."""
        return self.where(cond, other)

    # ------------------------------------------------------------------ in-place state (reference value.rs setters)
    @staticmethod
    def from_tensor(t, requires_grad: bool = False) -> "Value":
        return Value(t, requires_grad)

    @staticmethod
    def from_slice(data, shape, requires_grad: bool = False) -> "Value":
        return Value(torch.as_tensor(data, dtype=torch.float32).reshape(tuple(shape)), requires_grad)

    def set_data(self, t) -> None:
        """Replace the values in place (shape must match), outside the graph."""
        with torch.no_grad():
            self.tensor.copy_(_t(t))

    def set_name(self, name: str) -> "Value":
        self.name = name
        return self

    def set_requires_grad(self, flag: bool) -> "Value":
        if self.tensor.is_leaf:
            self.tensor.requires_grad_(flag)
        elif not flag:
            self.tensor = self.tensor.detach()
        return self

    def to_vec(self) -> list[float]:
        return [float(v) for v in self.tensor.detach().reshape(-1).cpu().tolist()]

    def avg_pool2d(self, k, stride=None):
        return Value._wrap(torch.nn.functional.avg_pool2d(self.tensor, k, stride), "avg_pool2d", self)


class NoGradGuard:
    """Disables gradient recording while alive (reference ``NoGradGuard``, value.rs:14-66)."""

    def __enter__(self):
        self._g = torch.no_grad()
        self._g.__enter__()
        return self

    def __exit__(self, *a):
        self._g.__exit__(*a)


def no_grad():
    return NoGradGuard()


def with_no_grad(fn, *args, **kw):
    with torch.no_grad():
        return fn(*args, **kw)


def is_grad_enabled() -> bool:
    return torch.is_grad_enabled()


def set_grad_enabled(flag: bool):
    """Context manager (or plain call) that turns gradient recording on or off."""
    return torch.set_grad_enabled(flag)


def with_enable_grad(fn, *args, **kw):
    with torch.enable_grad():
        return fn(*args, **kw)


def grad_of(v: Value):
    return v.grad()


def zero_grad_from(root: Value) -> None:
    """Clear the gradients of every leaf that ``root`` depends on."""
    seen, keep, stack = set(), [], [root.tensor.grad_fn]
    while stack:
        n = stack.pop()
        if n is None or id(n) in seen:
            continue
        seen.add(id(n))
        keep.append(n)  # node wrappers stay alive, so their ids are not reused during the walk
        var = getattr(n, "variable", None)
        if var is not None:
            var.grad = None
        stack.extend(p for p, _ in getattr(n, "next_functions", ()))
    if root.tensor.is_leaf:
        root.tensor.grad = None


def backward_from(v: Value) -> None:
    v.backward()


def backward_with_grad(v: Value, grad) -> None:
    v.backward(grad)
