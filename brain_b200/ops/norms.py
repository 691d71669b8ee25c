"""RMSNorm / LayerNorm ops (``csrc/norms.cu``) with autograd and an optional fused residual add.

``rms_norm(x, w, eps)`` follows the reference definition ``x * (mean(x^2) + eps)^-1/2 * w``
(crates/brain-transformer/src/ops.rs:103-131); ``layer_norm`` uses the biased variance with eps
inside the square root (crates/brain-transformer/src/ops.rs:57-101). ``add_rms_norm(x, r, w)``
returns ``(norm(x + r), x + r)`` like ``fused_add_rmsnorm`` (crates/brain-core/src/tensor/ops_fused.rs:77-125).

If the weight carries a ``main_grad`` buffer (flat gradient storage used by the data-parallel
engine), its gradient is accumulated there by the kernel and autograd receives ``None``.
"""
from __future__ import annotations

import torch

from .. import _native
from ._common import has_main_grad, main_grad_beta, ptr, rows2d, stream

_RMS, _LN = 0, 1


def _fwd(kind, x2, w, b, eps, res2=None):
    M, D = x2.shape
    y = torch.empty_like(x2)
    rstd = torch.empty(M, device=x2.device, dtype=torch.float32)
    mean = torch.empty(M, device=x2.device, dtype=torch.float32) if kind == _LN else None
    s = torch.empty_like(x2) if res2 is not None else None
    _native.call(
        "brain_norm_fwd", kind, x2.data_ptr(), x2.stride(0), ptr(res2), res2.stride(0) if res2 is not None else 0,
        w.data_ptr(), ptr(b), y.data_ptr(), y.stride(0), ptr(s), s.stride(0) if s is not None else 0,
        ptr(mean), rstd.data_ptr(), M, D, float(eps), stream(x2))
    return y, s, mean, rstd


def _bwd(kind, dy2, x2, w, b, mean, rstd, dres2=None):
    """Returns (dx, dw, db); dw/db are None when accumulated into main_grad."""
    M, D = x2.shape
    dx = torch.empty_like(x2)
    P = _native.fn("brain_norm_bwd_partials")(M)
    ws = torch.empty(2 * P * D, device=x2.device, dtype=torch.float32)
    use_main = has_main_grad(w)
    if use_main:
        dw = w.main_grad
        db = b.main_grad if (b is not None and has_main_grad(b)) else None
        dw_f32 = int(dw.dtype == torch.float32)
        bw = main_grad_beta(w)
        bb = main_grad_beta(b) if db is not None else bw
        if bw != bb:  # one accumulate flag covers both: clear the fresh one and accumulate into both
            (dw if bw == 0.0 else db).zero_()
            bw = 1.0
        acc = int(bw != 0.0)
    else:
        dw = torch.empty(D, device=x2.device, dtype=torch.float32)
        db = torch.empty(D, device=x2.device, dtype=torch.float32) if b is not None else None
        dw_f32, acc = 1, 0
    _native.call(
        "brain_norm_bwd", kind, dy2.data_ptr(), dy2.stride(0), x2.data_ptr(), x2.stride(0), w.data_ptr(),
        ptr(mean), rstd.data_ptr(), dx.data_ptr(), dx.stride(0), ptr(dres2), dres2.stride(0) if dres2 is not None else 0,
        dw.data_ptr(), ptr(db), dw_f32, acc, ws.data_ptr(), M, D, stream(x2))
    if use_main:
        return dx, None, None
    return dx, dw.to(w.dtype), (db.to(b.dtype) if db is not None else None)


class _NormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps, kind):
        x2 = rows2d(x)
        y, _, mean, rstd = _fwd(kind, x2, w, b, eps)
        ctx.save_for_backward(x2, w, b, mean, rstd)
        ctx.kind = kind
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, b, mean, rstd = ctx.saved_tensors
        dx, dw, db = _bwd(ctx.kind, rows2d(dy), x2, w, b, mean, rstd)
        return dx.view(ctx.shape), dw, db, None, None


class _AddNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, r, w, b, eps, kind):
        x2, r2 = rows2d(x), rows2d(r)
        y, s, mean, rstd = _fwd(kind, x2, w, b, eps, r2)
        ctx.save_for_backward(s, w, b, mean, rstd)
        ctx.kind = kind
        ctx.shape = x.shape
        return y.view(x.shape), s.view(x.shape)

    @staticmethod
    def backward(ctx, dy, ds):
        s, w, b, mean, rstd = ctx.saved_tensors
        ds2 = rows2d(ds) if ds is not None else None
        dx, dw, db = _bwd(ctx.kind, rows2d(dy), s, w, b, mean, rstd, ds2)
        dx = dx.view(ctx.shape)
        return dx, dx, dw, db, None, None


# ------------------------------------------------------------------ CPU oracle restatements
def rms_norm_ref(x, w, eps):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return y.to(x.dtype)


def layer_norm_ref(x, w, b, eps):
    xf = x.float()
    mu = xf.mean(-1, keepdim=True)
    var = (xf - mu).pow(2).mean(-1, keepdim=True)
    y = (xf - mu) * torch.rsqrt(var + eps) * w.float()
    if b is not None:
        y = y + b.float()
    return y.to(x.dtype)


# ------------------------------------------------------------------ public ops
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if x.is_cuda:
        return _NormFn.apply(x, w, None, eps, _RMS)
    return rms_norm_ref(x, w, eps)


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None, eps: float = 1e-5) -> torch.Tensor:
    if x.is_cuda:
        return _NormFn.apply(x, w, b, eps, _LN)
    return layer_norm_ref(x, w, b, eps)


def add_rms_norm(x, r, w, eps=1e-6):
    """(rms_norm(x + r), x + r) in one pass."""
    if x.is_cuda:
        return _AddNormFn.apply(x, r, w, None, eps, _RMS)
    s = x + r
    return rms_norm_ref(s, w, eps), s


def add_layer_norm(x, r, w, b=None, eps=1e-5):
    if x.is_cuda:
        return _AddNormFn.apply(x, r, w, b, eps, _LN)
    s = x + r
    return layer_norm_ref(s, w, b, eps), s


def fused_layer_norm(x, w, b=None, eps=1e-5):
    """LayerNorm with the one-pass variance of the reference's fused variant: var = max(E[x^2] - E[x]^2, 0)
    (crates/brain-core/src/tensor/ops_fused.rs:43-70). On CUDA tensors the LayerNorm kernel runs; it takes
    the two-pass variance, which equals the one-pass form in exact arithmetic and does not cancel. On the
    CPU float64 inputs are computed in float64 (the reference's precision), others in float32."""
    if x.is_cuda:
        return layer_norm(x, w, b, eps)
    ct = torch.float64 if x.dtype == torch.float64 else torch.float32
    xf = x.to(ct)
    mu = xf.mean(-1, keepdim=True)
    var = (xf.pow(2).mean(-1, keepdim=True) - mu.pow(2)).clamp_min(0.0)
    y = (xf - mu) * torch.rsqrt(var + eps) * w.to(ct)
    if b is not None:
        y = y + b.to(ct)
    return y.to(x.dtype)
