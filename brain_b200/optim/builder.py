"""Fluent optimizer construction and parameter groups with the reference's names: ``OptimizerKind``,
``OptimizerBuilder`` (``OptimizerBuilder().adamw().lr(3e-4).betas(0.9, 0.95).build(params)``),
``ParamGroup`` / ``ParamGroupConfig`` (per-group lr, betas, weight decay, lr multiplier, freezing) and
``GradEntry`` (a gradient with its norm and non-finite flag).

Reference: crates/brain-optim/src/builder.rs:8-170 (kinds, defaults lr 1e-3, betas 0.9/0.999,
eps 1e-8; ``lion()`` switches the betas to 0.9/0.99), optimizer/param_group.rs:9-135.

``build`` returns this package's optimizers (the fused AdamW / SGD kernels on CUDA parameters), so a
built optimizer is the same object a direct constructor call gives.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field

import torch

from . import optimizers as _o
from . import schedulers as _s


class OptimizerKind(enum.Enum):
    Adam = "adam"
    AdamW = "adamw"
    Sgd = "sgd"
    SgdNesterov = "sgd_nesterov"
    Rmsprop = "rmsprop"
    Adagrad = "adagrad"
    Adadelta = "adadelta"
    Lamb = "lamb"
    Lion = "lion"
    RAdam = "radam"
    Adafactor = "adafactor"
    NovoGrad = "novograd"


@dataclass
class ParamGroupConfig:
    name: str = "default"
    lr: float = 1e-3
    weight_decay: float = 0.0
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    lr_multiplier: float = 1.0
    is_frozen: bool = False
    dampening: float = 0.0


@dataclass
class ParamGroup:
    """A group of parameters (tensors) with its own hyper-parameters. ``effective_lr`` is
    lr x lr_multiplier, or 0 for a frozen group; ``as_dict`` is the group an optimizer receives."""
    params: list
    lr: float = 1e-3
    weight_decay: float = 0.0
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    lr_multiplier: float = 1.0
    is_frozen: bool = False
    name: str = "default"
    options: dict = field(default_factory=dict)
    initial_lr: float | None = None

    def __post_init__(self):
        self.params = list(self.params)
        if self.initial_lr is None:
            self.initial_lr = self.lr

    @classmethod
    def from_config(cls, params, config: ParamGroupConfig) -> "ParamGroup":
        return cls(params, config.lr, config.weight_decay, config.beta1, config.beta2, config.eps,
                   config.lr_multiplier, config.is_frozen, config.name)

    def with_weight_decay(self, wd: float) -> "ParamGroup":
        self.weight_decay = wd
        return self

    def with_betas(self, b1: float, b2: float) -> "ParamGroup":
        self.beta1, self.beta2 = b1, b2
        return self

    def with_name(self, name: str) -> "ParamGroup":
        self.name = name
        return self

    def with_option(self, key: str, val: float) -> "ParamGroup":
        self.options[key] = val
        return self

    def effective_lr(self) -> float:
        return 0.0 if self.is_frozen else self.lr * self.lr_multiplier

    def as_dict(self, with_betas: bool = True) -> dict:
        d = {"params": self.params, "lr": self.effective_lr(), "weight_decay": self.weight_decay,
             "name": self.name, **self.options}
        if with_betas:  # Adam-family groups; the others keep their own eps defaults
            d["betas"], d["eps"] = (self.beta1, self.beta2), self.eps
        return d


class GradEntry:
    """A parameter's gradient with its L2 norm and whether any element is inf/nan (one reduction)."""

    def __init__(self, param_id: int, grad: torch.Tensor):
        self.param_id, self.grad = param_id, grad
        g = grad.detach().float()
        self.norm = float(torch.linalg.vector_norm(g)) if g.numel() else 0.0
        self.has_nan = not bool(torch.isfinite(g).all()) if g.numel() else False


_BETAS = {OptimizerKind.Adam, OptimizerKind.AdamW, OptimizerKind.Lamb, OptimizerKind.Lion, OptimizerKind.RAdam,
          OptimizerKind.NovoGrad}


class OptimizerBuilder:
    def __init__(self):
        self.kind = OptimizerKind.Adam
        self._lr, self._wd, self.beta1, self.beta2, self._eps = 1e-3, 0.0, 0.9, 0.999, 1e-8
        self._momentum, self.dampening, self._nesterov, self._amsgrad, self.centered = 0.0, 0.0, False, False, False
        self.param_groups: list[ParamGroup] = []
        self.extra_options: dict = {}

    def _k(self, kind):
        self.kind = kind
        return self

    def adam(self):
        return self._k(OptimizerKind.Adam)

    def adamw(self):
        return self._k(OptimizerKind.AdamW)

    def sgd(self):
        return self._k(OptimizerKind.Sgd)

    def lion(self):
        self.beta1, self.beta2 = 0.9, 0.99
        return self._k(OptimizerKind.Lion)

    def lamb(self):
        return self._k(OptimizerKind.Lamb)

    def rmsprop(self):
        return self._k(OptimizerKind.Rmsprop)

    def adagrad(self):
        return self._k(OptimizerKind.Adagrad)

    def adadelta(self):
        return self._k(OptimizerKind.Adadelta)

    def radam(self):
        return self._k(OptimizerKind.RAdam)

    def adafactor(self):
        return self._k(OptimizerKind.Adafactor)

    def novograd(self):
        return self._k(OptimizerKind.NovoGrad)

    def lr(self, lr: float):
        self._lr = lr
        return self

    def weight_decay(self, wd: float):
        self._wd = wd
        return self

    def betas(self, b1: float, b2: float):
        self.beta1, self.beta2 = b1, b2
        return self

    def eps(self, eps: float):
        self._eps = eps
        return self

    def momentum(self, m: float):
        self._momentum = m
        return self

    def nesterov(self, n: bool):
        self._nesterov = n
        return self

    def amsgrad(self, a: bool):
        self._amsgrad = a
        return self

    def add_param_group(self, group: ParamGroup):
        self.param_groups.append(group)
        return self

    def build(self, params=None) -> _o.Optimizer:
        """The optimizer over ``params`` (tensors or group dicts) and/or the added ParamGroups."""
        k = self.kind
        groups = []
        if params is not None:
            params = list(params)
            groups += params if params and isinstance(params[0], dict) else ([{"params": params}] if params else [])
        groups += [g.as_dict(k in _BETAS) for g in self.param_groups]
        betas, lr, wd, eps = (self.beta1, self.beta2), self._lr, self._wd, self._eps
        if k is OptimizerKind.Adam:
            return _o.Adam(groups, lr=lr, betas=betas, eps=eps, weight_decay=wd, amsgrad=self._amsgrad)
        if k is OptimizerKind.AdamW:
            return _o.AdamW(groups, lr=lr, betas=betas, eps=eps, weight_decay=wd, amsgrad=self._amsgrad)
        if k in (OptimizerKind.Sgd, OptimizerKind.SgdNesterov):
            nest = self._nesterov or k is OptimizerKind.SgdNesterov
            mom = self._momentum if self._momentum or not nest else 0.9
            return _o.SGD(groups, lr=lr, momentum=mom, dampening=self.dampening, weight_decay=wd, nesterov=nest)
        if k is OptimizerKind.Rmsprop:
            return _o.RMSprop(groups, lr=lr, eps=eps, weight_decay=wd, momentum=self._momentum, centered=self.centered,
                              **self.extra_options)
        if k is OptimizerKind.Adagrad:
            return _o.Adagrad(groups, lr=lr, weight_decay=wd, **self.extra_options)
        if k is OptimizerKind.Adadelta:
            return _o.Adadelta(groups, lr=lr, weight_decay=wd, **self.extra_options)
        if k is OptimizerKind.Adafactor:
            return _o.Adafactor(groups, lr=lr, weight_decay=wd, **self.extra_options)
        cls = {OptimizerKind.Lamb: _o.Lamb, OptimizerKind.RAdam: _o.RAdam, OptimizerKind.NovoGrad: _o.NovoGrad}.get(k)
        if cls is not None:
            return cls(groups, lr=lr, betas=betas, eps=eps, weight_decay=wd)
        if k is OptimizerKind.Lion:
            return _o.Lion(groups, lr=lr, betas=betas, weight_decay=wd)
        raise ValueError(f"unknown optimizer kind {k}")


# The reference's spellings of classes that exist here under the PyTorch-style names.
Rmsprop = _o.RMSprop
SophiaG = _o.Sophia
SwAOptimizer = _o.SWA
ModelEma = _o.EMA
LrFinder = _s.LRFinder
LrScheduler = _s.LRScheduler


def SgdNesterov(params, lr: float = 0.01, momentum: float = 0.9, weight_decay: float = 0.0) -> _o.SGD:
    return _o.SGD(params, lr=lr, momentum=momentum, weight_decay=weight_decay, nesterov=True)
