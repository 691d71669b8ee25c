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


class CheckpointPolicy:
    """Which layers recompute their activations in backward: ``"none"``, ``"all"``, ``"sqrt"`` (every
    round(sqrt(L))-th layer, ``BudgetCheckpoint``) or ``"every:k"`` (reference ``CheckpointPolicy``,
    crates/brain-autograd/src/checkpoint/mod.rs:15-37)."""

    def __init__(self, kind: str = "none"):
        self.kind = kind

    def mask(self, num_layers: int) -> list[bool]:
        if self.kind == "all":
            return [True] * num_layers
        if self.kind == "sqrt":
            return BudgetCheckpoint(num_layers).mask(num_layers)
        if self.kind.startswith("every:"):
            k = max(1, int(self.kind.split(":", 1)[1]))
            return [i % k == 0 for i in range(num_layers)]
        return [False] * num_layers


class CpuOffloader:
    """Context manager that moves the activations autograd saves for backward to pinned host memory
    (copied on a side stream) and brings them back when backward needs them (reference ``CpuOffloader``,
    crates/brain-autograd/src/cpu_offload.rs). Tensors smaller than ``min_bytes`` stay on the device.
    Trades PCIe / C2C bandwidth for HBM when activations do not fit."""

    def __init__(self, min_bytes: int = 1 << 20):
        self.min_bytes = min_bytes
        self.offloaded = 0
        self._ctx = None

    def _pack(self, t: torch.Tensor):
        if not t.is_cuda or t.numel() * t.element_size() < self.min_bytes:
            return t
        stream = torch.cuda.current_stream(t.device)
        side = self._side(t.device)
        side.wait_stream(stream)
        host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        with torch.cuda.stream(side):
            host.copy_(t, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(side)
        t.record_stream(side)
        self.offloaded += t.numel() * t.element_size()
        return (host, t.device, ev)

    def _unpack(self, packed):
        if isinstance(packed, torch.Tensor):
            return packed
        host, dev, ev = packed
        ev.synchronize()
        return host.to(dev, non_blocking=True)

    def _side(self, dev):
        if not hasattr(self, "_streams"):
            self._streams = {}
        if dev not in self._streams:
            self._streams[dev] = torch.cuda.Stream(dev)
        return self._streams[dev]

    def __enter__(self):
        self._ctx = torch.autograd.graph.saved_tensors_hooks(self._pack, self._unpack)
        self._ctx.__enter__()
        return self

    def __exit__(self, *exc):
        self._ctx.__exit__(*exc)
        return False


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
