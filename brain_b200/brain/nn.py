"""``brain.nn``: Module discovery of parameters, Linear, Conv2d, LayerNorm, MSELoss, CrossEntropyLoss
(reference python/brain/nn/__init__.py and crates/brain-python/src/nn.rs)."""
from __future__ import annotations

import math

import torch

from ._core import Tensor, Value, _unwrap


class Module:
    """Base class: ``parameters()`` collects the gradient-tracking Values stored on the object, in
    sub-modules and in lists of either, in attribute order."""

    def __init__(self):
        pass

    def __call__(self, *args, **kw):
        return self.forward(*args, **kw)

    def forward(self, *args, **kw):
        raise NotImplementedError("forward method must be implemented by subclass")

    def parameters(self) -> list:
        out = []

        def visit(v):
            if isinstance(v, Module):
                out.extend(v.parameters())
            elif isinstance(v, Value) and v.requires_grad:
                out.append(v)
            elif isinstance(v, (list, tuple)):
                for x in v:
                    visit(x)
        for v in self.__dict__.values():
            visit(v)
        return out

    def zero_grad(self) -> None:
        for p in self.parameters():
            p.zero_grad()

    def to(self, device) -> "Module":
        for k, v in list(self.__dict__.items()):
            if isinstance(v, (Value, Module)):
                setattr(self, k, v.to(device))
        return self


def _kaiming_uniform(shape, fan_in) -> torch.Tensor:
    bound = 1.0 / math.sqrt(fan_in)
    return torch.empty(shape).uniform_(-bound, bound)


class Linear(Module):
    """y = x Wᵀ + b with W [out, in]; bf16 CUDA inputs run the framework's tcgen05 GEMM."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.weight = Value(_kaiming_uniform((out_features, in_features), in_features), requires_grad=True)
        self.bias = Value(torch.zeros(out_features), requires_grad=True) if bias else None

    def forward(self, x):
        xt = _unwrap(x)
        w = self.weight._t
        b = self.bias._t if self.bias is not None else None
        if xt.is_cuda and xt.dtype == torch.bfloat16:
            from .. import ops
            y = ops.linear(xt, w.to(torch.bfloat16), None if b is None else b.to(torch.bfloat16))
        else:
            y = torch.nn.functional.linear(xt.to(w.dtype), w, b)
        return Value._of(y)


class Conv2d(Module):
    """Stride 1 and "same" padding (k // 2) by default, so an 8x8 input with k = 3 stays 8x8."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, bias: bool = True, stride: int = 1,
                 padding: int | None = None):
        super().__init__()
        k = kernel_size
        self.stride, self.padding = stride, k // 2 if padding is None else padding
        self.weight = Value(_kaiming_uniform((out_channels, in_channels, k, k), in_channels * k * k),
                            requires_grad=True)
        self.bias = Value(torch.zeros(out_channels), requires_grad=True) if bias else None

    def forward(self, x):
        xt = _unwrap(x)
        return Value._of(torch.nn.functional.conv2d(xt.to(self.weight._t.dtype), self.weight._t,
                                                    None if self.bias is None else self.bias._t, self.stride,
                                                    self.padding))


class LayerNorm(Module):
    def __init__(self, normalized_shape, eps: float = 1e-5):
        super().__init__()
        shape = [normalized_shape] if isinstance(normalized_shape, int) else list(normalized_shape)
        self.shape, self.eps = shape, eps
        self.weight = Value(torch.ones(shape), requires_grad=True)
        self.bias = Value(torch.zeros(shape), requires_grad=True)

    def forward(self, x):
        xt = _unwrap(x)
        return Value._of(torch.nn.functional.layer_norm(xt.to(self.weight._t.dtype), self.shape, self.weight._t,
                                                        self.bias._t, self.eps))


class MSELoss(Module):
    def forward(self, pred, target):
        return Value._of(torch.nn.functional.mse_loss(_unwrap(pred), _unwrap(target).to(_unwrap(pred).dtype)).reshape(1))


class CrossEntropyLoss(Module):
    """Logits [N, C] and integer class targets [N] (or their float encoding); mean over N."""

    def __init__(self, label_smoothing: float = 0.0):
        super().__init__()
        self.label_smoothing = label_smoothing

    def forward(self, logits, targets):
        lt, tt = _unwrap(logits), _unwrap(targets)
        if tt.is_floating_point() and tt.shape == lt.shape:  # probabilities / one-hot
            loss = torch.nn.functional.cross_entropy(lt, tt, label_smoothing=self.label_smoothing)
        else:
            loss = torch.nn.functional.cross_entropy(lt, tt.long().reshape(-1), label_smoothing=self.label_smoothing)
        return Value._of(loss.reshape(1))


__all__ = ["Module", "Linear", "Conv2d", "LayerNorm", "MSELoss", "CrossEntropyLoss", "Tensor", "Value"]
