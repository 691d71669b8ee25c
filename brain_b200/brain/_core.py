"""``Tensor`` and ``Value`` of the reference's Python API (see the package docstring)."""
from __future__ import annotations

import torch

DTYPE = torch.float32


def _as_torch(data, shape=None, requires_grad: bool = False) -> torch.Tensor:
    if isinstance(data, (Tensor, Value)):
        t = data._t.detach().clone()
    elif isinstance(data, torch.Tensor):
        t = data.detach().clone()
    else:
        t = torch.tensor(data, dtype=DTYPE)
    if not t.is_floating_point():
        t = t.to(DTYPE)
    if shape is not None:
        shape = [int(d) for d in shape]
        n = 1
        for d in shape:
            n *= d
        if n != t.numel():
            raise ValueError(f"data has {t.numel()} elements but shape {shape} needs {n}")
        t = t.reshape(shape)
    if requires_grad:
        t.requires_grad_(True)
    return t


def _unwrap(x):
    if isinstance(x, (Tensor, Value)):
        return x._t
    if isinstance(x, torch.Tensor):
        return x
    return torch.tensor(x, dtype=DTYPE)


class _Base:
    __slots__ = ("_t",)

    @property
    def shape(self) -> list[int]:
        return list(self._t.shape)

    @property
    def ndim(self) -> int:
        return self._t.dim()

    @property
    def numel(self) -> int:
        return self._t.numel()

    @property
    def device(self) -> str:
        return str(self._t.device)

    def to_list(self) -> list[float]:
        return [float(v) for v in self._t.detach().reshape(-1).cpu().tolist()]

    def item(self) -> float:
        if self._t.numel() != 1:
            raise ValueError(f"item() needs exactly one element, tensor has {self._t.numel()}")
        return float(self._t.detach().reshape(-1)[0])

    def torch(self) -> torch.Tensor:
        return self._t

    def __repr__(self):
        return f"{type(self).__name__}(shape={self.shape}, data={self.to_list()[:8]}{'...' if self.numel > 8 else ''})"


class Tensor(_Base):
    """N-D array without gradient tracking."""

    def __init__(self, data, shape=None):
        self._t = _as_torch(data, shape)

    @classmethod
    def _of(cls, t: torch.Tensor) -> "Tensor":
        o = cls.__new__(cls)
        o._t = t.detach()
        return o

    def to(self, device) -> "Tensor":
        return Tensor._of(self._t.to(device))

    def reshape(self, shape) -> "Tensor":
        return Tensor._of(self._t.reshape([int(d) for d in shape]))

    def transpose(self, a: int, b: int) -> "Tensor":
        return Tensor._of(self._t.transpose(a, b).contiguous())

    def sum(self) -> "Tensor":
        return Tensor._of(self._t.sum().reshape(1))

    def mean(self) -> "Tensor":
        return Tensor._of(self._t.mean().reshape(1))

    def _bin(self, o, f):
        if isinstance(o, Value):
            return NotImplemented
        return Tensor._of(f(self._t, _unwrap(o)))

    def __add__(self, o):
        return self._bin(o, torch.add)

    def __sub__(self, o):
        return self._bin(o, torch.sub)

    def __mul__(self, o):
        return self._bin(o, torch.mul)

    def __truediv__(self, o):
        return self._bin(o, torch.div)

    def __matmul__(self, o):
        return self._bin(o, torch.matmul)

    __radd__ = __add__
    __rmul__ = __mul__

    def __rsub__(self, o):
        return Tensor._of(torch.sub(_unwrap(o), self._t))

    def __neg__(self):
        return Tensor._of(-self._t)


class Value(_Base):
    """Autograd node: ``grad`` is a ``Tensor`` after ``backward()``, ``None`` before."""

    def __init__(self, data, shape=None, requires_grad: bool = False):
        self._t = _as_torch(data, shape, requires_grad)

    @classmethod
    def _of(cls, t: torch.Tensor) -> "Value":
        o = cls.__new__(cls)
        o._t = t
        return o

    @property
    def requires_grad(self) -> bool:
        return self._t.requires_grad

    @property
    def grad(self):
        g = self._t.grad
        return None if g is None else Tensor._of(g)

    @property
    def data(self) -> Tensor:
        return Tensor._of(self._t)

    def zero_grad(self) -> None:
        self._t.grad = None

    def backward(self) -> None:
        self._t.backward(torch.ones_like(self._t))

    def to(self, device) -> "Value":
        t = self._t.detach().to(device)
        if self._t.requires_grad:
            t.requires_grad_(True)
        return Value._of(t)

    def _bin(self, o, f):
        return Value._of(f(self._t, _unwrap(o)))

    def __add__(self, o):
        return self._bin(o, torch.add)

    def __sub__(self, o):
        return self._bin(o, torch.sub)

    def __mul__(self, o):
        return self._bin(o, torch.mul)

    def __truediv__(self, o):
        return self._bin(o, torch.div)

    def __matmul__(self, o):
        return self._bin(o, torch.matmul)

    def __radd__(self, o):
        return Value._of(torch.add(_unwrap(o), self._t))

    def __rsub__(self, o):
        return Value._of(torch.sub(_unwrap(o), self._t))

    def __rmul__(self, o):
        return Value._of(torch.mul(_unwrap(o), self._t))

    def __neg__(self):
        return Value._of(-self._t)

    def relu(self):
        return Value._of(torch.relu(self._t))

    def sigmoid(self):
        return Value._of(torch.sigmoid(self._t))

    def tanh(self):
        return Value._of(torch.tanh(self._t))

    def exp(self):
        return Value._of(torch.exp(self._t))

    def log(self):
        return Value._of(torch.log(self._t))

    def sum(self):
        return Value._of(self._t.sum().reshape(1))

    def mean(self):
        return Value._of(self._t.mean().reshape(1))

    def reshape(self, shape):
        return Value._of(self._t.reshape([int(d) for d in shape]))

    def transpose(self, a: int, b: int):
        return Value._of(self._t.transpose(a, b))


def zeros(shape) -> Tensor:
    return Tensor._of(torch.zeros([int(d) for d in shape], dtype=DTYPE))


def ones(shape) -> Tensor:
    return Tensor._of(torch.ones([int(d) for d in shape], dtype=DTYPE))


def tensor(data, shape=None) -> Tensor:
    return Tensor(data, shape)
