"""Functional transforms and gradient utilities.

Reference: ``grad``, ``value_and_grad``, ``vjp``, ``jvp``, ``jacobian``, ``hessian``
(crates/brain-autograd/src/graph_closure.rs:11-146); activation checkpointing
(checkpoint/selective.rs:9-32, ``BudgetCheckpoint`` sqrt(L) policy); dynamic loss scaling
``GradScaler`` (engine/mixed.rs:9-97: init 65536, x2 every 2000 finite steps, x0.5 on inf/nan);
``parallel_backward`` (engine/parallel.rs:25-62). The transforms are exact (``torch.func``),
where the reference's hessian is a finite difference of gradients.
"""
from __future__ import annotations

import math

import torch
import torch.utils.checkpoint as _ckpt

from .value import Value


def _unwrap(fn):
    def f(*xs):
        out = fn(*[Value(x) if not isinstance(x, Value) else x for x in xs])
        return out.tensor if isinstance(out, Value) else out
    return f


def grad(fn, argnums=0):
    """Returns a function computing d fn / d args[argnums] (fn returns a scalar)."""
    g = torch.func.grad(_unwrap(fn), argnums=argnums)
    return lambda *xs: g(*[x.tensor if isinstance(x, Value) else x for x in xs])


def value_and_grad(fn, argnums=0):
    g = torch.func.grad_and_value(_unwrap(fn), argnums=argnums)

    def f(*xs):
        gr, val = g(*[x.tensor if isinstance(x, Value) else x for x in xs])
        return val, gr
    return f


def vjp(fn, x, v):
    """(fn(x), v^T J)."""
    out, pull = torch.func.vjp(_unwrap(fn), x.tensor if isinstance(x, Value) else x)
    return out, pull(v)[0]


def jvp(fn, x, t):
    """(fn(x), J t)."""
    return torch.func.jvp(_unwrap(fn), (x.tensor if isinstance(x, Value) else x,), (t,))


def jacobian(fn, x):
    return torch.func.jacrev(_unwrap(fn))(x.tensor if isinstance(x, Value) else x)


def hessian(fn, x):
    return torch.func.hessian(_unwrap(fn))(x.tensor if isinstance(x, Value) else x)


def grad_and_hess(fn, x):
    xt = x.tensor if isinstance(x, Value) else x
    return torch.func.grad(_unwrap(fn))(xt), torch.func.hessian(_unwrap(fn))(xt)


def numeric_grad(fn, x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Central finite differences in float64 (the reference grad-check harness, grad_check.rs:16-70)."""
    x = x.detach().double().clone()
    g = torch.zeros_like(x)
    flat, gflat = x.view(-1), g.view(-1)
    for i in range(flat.numel()):
        old = flat[i].item()
        flat[i] = old + eps
        fp = float(fn(x))
        flat[i] = old - eps
        fm = float(fn(x))
        flat[i] = old
        gflat[i] = (fp - fm) / (2 * eps)
    return g


def checkpoint(fn, *inputs, use_reentrant: bool = False):
    """Recompute ``fn`` in backward instead of storing its activations."""
    if not torch.is_grad_enabled():
        return fn(*inputs)
    return _ckpt.checkpoint(fn, *inputs, use_reentrant=use_reentrant)


class BudgetCheckpoint:
    """Checkpoint every k-th of L layers with k = round(sqrt(L)) (reference sqrt(L) mask)."""

    def __init__(self, num_layers: int):
        self.every = max(1, round(math.sqrt(num_layers)))

    def mask(self, num_layers: int) -> list[bool]:
        return [i % self.every == 0 for i in range(num_layers)]


class GradScaler:
    """Dynamic loss scaling: scale the loss, unscale grads, skip non-finite steps and back off."""

    def __init__(self, init_scale: float = 65536.0, growth_factor: float = 2.0, backoff_factor: float = 0.5,
                 growth_interval: int = 2000, enabled: bool = True):
        self.scale = float(init_scale)
        self.growth_factor, self.backoff_factor = growth_factor, backoff_factor
        self.growth_interval = growth_interval
        self.enabled = enabled
        self._good = 0
        self.skipped = 0

    def scale_loss(self, loss):
        return loss * self.scale if self.enabled else loss

    def inv_scale(self) -> float:
        return 1.0 / self.scale if self.enabled else 1.0

    def update(self, found_inf: bool) -> None:
        if not self.enabled:
            return
        if found_inf:
            self.scale *= self.backoff_factor
            self._good = 0
            self.skipped += 1
        else:
            self._good += 1
            if self._good % self.growth_interval == 0:
                self.scale *= self.growth_factor

    def state_dict(self):
        return {"scale": self.scale, "good": self._good, "skipped": self.skipped}

    def load_state_dict(self, sd):
        self.scale, self._good, self.skipped = sd["scale"], sd["good"], sd["skipped"]


def parallel_backward(losses: list[Value]) -> None:
    """Backward of several independent losses (summed in one engine pass)."""
    total = None
    for l in losses:
        t = l.tensor if isinstance(l, Value) else l
        total = t if total is None else total + t
    if total is not None:
        total.backward()
