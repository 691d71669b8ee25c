"""Flat-buffer optimizer kernels (``csrc/optim.cu``): fused AdamW / SGD, squared norms, scaling.

All functions take flat (1-D, contiguous) buffers: float32 master weights and moments, a bf16 or
float32 gradient, and optionally a bf16 compute copy of the weights written in the same pass.
``found_inf`` is a device int32 flag; when non-zero the update kernels skip the step, which is how a
non-finite gradient is handled under dynamic loss scaling.
"""
from __future__ import annotations

import torch

from .. import _native
from ._common import ptr, stream


def adamw_(p, m, v, g, *, lr, beta1, beta2, eps, weight_decay, step, grad_scale=1.0, p16=None, vmax=None,
           found_inf=None, bias_correction=True, coef=None):
    """One AdamW step (reference order: decay, moments, bias-corrected update) over flat buffers.

    ``found_inf`` (device int32 scalar): skip the step when non-zero. ``coef`` (device float32 scalar):
    an extra factor on the gradient, e.g. the global-norm clipping coefficient of ``step_guard``."""
    bc1 = 1.0 - beta1 ** step if bias_correction else 1.0
    bc2 = 1.0 - beta2 ** step if bias_correction else 1.0
    if p.is_cuda:
        _native.call("brain_adamw", p.data_ptr(), m.data_ptr(), v.data_ptr(), ptr(vmax), g.data_ptr(),
                     int(g.dtype == torch.float32), ptr(p16), p.numel(), float(lr), float(beta1), float(beta2),
                     float(eps), float(weight_decay), float(bc1), float(bc2), float(grad_scale), int(vmax is not None),
                     ptr(found_inf), ptr(coef), stream(p))
        return
    if found_inf is not None and int(found_inf.item()) != 0:
        return
    gf = g.float() * grad_scale
    if coef is not None:
        gf = gf * coef
    p.mul_(1.0 - lr * weight_decay)
    m.mul_(beta1).add_(gf, alpha=1.0 - beta1)
    v.mul_(beta2).addcmul_(gf, gf, value=1.0 - beta2)
    vh = v
    if vmax is not None:
        torch.maximum(vmax, v, out=vmax)
        vh = vmax
    p.sub_(lr * (m / bc1) / ((vh / bc2).sqrt() + eps))
    if p16 is not None:
        p16.copy_(p)


def sgd_(p, buf, g, *, lr, momentum=0.0, dampening=0.0, weight_decay=0.0, nesterov=False, first=False,
         grad_scale=1.0, p16=None, found_inf=None):
    if p.is_cuda:
        _native.call("brain_sgd", p.data_ptr(), ptr(buf), g.data_ptr(), int(g.dtype == torch.float32), ptr(p16),
                     p.numel(), float(lr), float(momentum), float(dampening), float(weight_decay), int(nesterov),
                     int(first), float(grad_scale), ptr(found_inf), stream(p))
        return
    if found_inf is not None and int(found_inf.item()) != 0:
        return
    d = g.float() * grad_scale + weight_decay * p
    if momentum != 0.0:
        if first:
            buf.copy_(d)
        else:
            buf.mul_(momentum).add_(d, alpha=1.0 - dampening)
        d = d + momentum * buf if nesterov else buf
    p.sub_(lr * d)
    if p16 is not None:
        p16.copy_(p)


def sumsq(g, scale=1.0, out=None, accumulate=False, found_inf=None):
    """sum((scale*g)^2) into a device float32 scalar; sets found_inf on a non-finite element."""
    if out is None:
        out = torch.zeros(1, device=g.device, dtype=torch.float32)
    if g.is_cuda:
        ws = torch.empty(1024, device=g.device, dtype=torch.float32)
        _native.call("brain_sumsq", g.data_ptr(), int(g.dtype == torch.float32), g.numel(), float(scale),
                     out.data_ptr(), int(accumulate), ptr(found_inf), ws.data_ptr(), stream(g))
        return out
    gf = g.float() * scale
    s = gf.pow(2).sum().reshape(1)
    out.copy_(out + s if accumulate else s)
    if found_inf is not None and not torch.isfinite(gf).all():
        found_inf.fill_(1)
    return out


def grad_stats(g, scale=1.0, stats=None, accumulate=False):
    """stats[0:2] (+)= (sum((scale*g)^2), 1.0 if any scale*g is non-finite) as a float32 device vector."""
    if stats is None:
        stats = torch.zeros(2, device=g.device, dtype=torch.float32)
    if g.is_cuda:
        ws = torch.empty(2048, device=g.device, dtype=torch.float32)
        _native.call("brain_grad_stats", g.data_ptr(), int(g.dtype == torch.float32), g.numel(), float(scale),
                     stats.data_ptr(), int(accumulate), ws.data_ptr(), stream(g))
        return stats
    gf = g.float() * scale
    new = torch.stack([gf.pow(2).sum(), (~torch.isfinite(gf)).any().float()])
    stats.copy_(stats + new if accumulate else new)
    return stats


def step_guard(stats, max_norm=0.0, found_inf=None, coef=None):
    """From globally reduced ``grad_stats``: found_inf (int32, 1 = skip the step) and the clip
    coefficient min(1, max_norm / (norm + 1e-6)) (1 when max_norm <= 0 or the step is skipped)."""
    if found_inf is None:
        found_inf = torch.zeros(1, device=stats.device, dtype=torch.int32)
    if coef is None:
        coef = torch.ones(1, device=stats.device, dtype=torch.float32)
    if stats.is_cuda:
        _native.call("brain_step_guard", stats.data_ptr(), float(max_norm), found_inf.data_ptr(), coef.data_ptr(),
                     stream(stats))
        return found_inf, coef
    sq = float(stats[0])
    bad = float(stats[1]) != 0.0 or not torch.isfinite(stats[0])
    found_inf.fill_(1 if bad else 0)
    coef.fill_(min(1.0, max_norm / (sq ** 0.5 + 1e-6)) if (max_norm > 0 and not bad) else 1.0)
    return found_inf, coef


def scale_(x, s):
    """x *= s where s is a python float or a device float32 scalar tensor."""
    if x.is_cuda:
        sp = s.data_ptr() if isinstance(s, torch.Tensor) else None
        sc = 1.0 if isinstance(s, torch.Tensor) else float(s)
        _native.call("brain_scale", x.data_ptr(), int(x.dtype == torch.float32), x.numel(), sp, sc, stream(x))
        return x
    x.mul_(s.to(x.dtype) if isinstance(s, torch.Tensor) else s)
    return x


def clip_coef(sq, max_norm):
    """Device scalar min(1, max_norm / (sqrt(sq) + 1e-6))."""
    out = torch.empty(1, device=sq.device, dtype=torch.float32)
    if sq.is_cuda:
        _native.call("brain_clip_coef", sq.data_ptr(), float(max_norm), out.data_ptr(), stream(sq))
        return out
    out.copy_(torch.clamp(max_norm / (sq.sqrt() + 1e-6), max=1.0))
    return out
