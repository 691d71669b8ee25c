"""Linear layers on the tcgen05 GEMM, with gradient accumulation into flat ``main_grad`` buffers.

``linear(x, w, b, residual)`` computes ``x @ w.T (+ b) (+ residual)`` in one GEMM (bias and residual
are epilogue adds). Backward: ``dx = dy @ w`` and ``dw = dy.T @ x`` both read their transposed
operands in place. When ``w`` has a ``main_grad`` attribute (a view into the flat gradient buffer of
the data-parallel engine / fused optimizer) the weight gradient GEMM accumulates straight into it
(``beta = 1``) and autograd gets ``None`` — no separate gradient tensor, no extra add.

Fused variants used by the transformer blocks keep activation memory low by recomputing cheap
elementwise producers in the backward pass:
* ``norm_linear``: ``rms_norm(x) @ w.T`` saving only x (the normalised input is recomputed);
* ``swiglu_linear``: ``swiglu(gu) @ w.T (+ residual)`` saving only gu.
Reference: brain-nn Linear ``x·Wᵀ + b`` (crates/brain-nn/src/layers/linear.rs:13-63).
"""
from __future__ import annotations

import torch

from .activations import swiglu_bwd_only, swiglu_fwd_only
from .gemm import gemm, gemm_rope
from .rope import apply_rope_
from ._common import has_main_grad, main_grad_beta, rows2d
from .. import _native
from . import norms as _norms


def _wgrad(dy2, x2, w):
    """Weight gradient dy^T x: into w.main_grad (returns None) or as a new tensor."""
    if has_main_grad(w):
        gemm(dy2, x2, trans_a=True, out=w.main_grad, beta=main_grad_beta(w))
        return None
    return gemm(dy2, x2, trans_a=True, out_dtype=torch.float32).to(w.dtype)


def _colsum_ok(dy2, out):
    return (dy2.is_cuda and dy2.dtype == torch.bfloat16 and dy2.stride(1) == 1 and dy2.size(1) % 8 == 0
            and dy2.stride(0) % 8 == 0 and dy2.data_ptr() % 16 == 0 and out.is_contiguous()
            and out.dtype in (torch.bfloat16, torch.float32))


def colsum_(dy2, out, accumulate=False):
    """out (+)= dy2.sum(0) with f32 accumulation on the native column-sum kernel (bias gradients)."""
    M, N = dy2.shape
    P = _native.fn("brain_colsum_partials")(M)
    ws = torch.empty(P * N, device=dy2.device, dtype=torch.float32)
    _native.call("brain_colsum_bf16", dy2.data_ptr(), dy2.stride(0), M, N, out.data_ptr(),
                 int(out.dtype == torch.float32), int(accumulate), ws.data_ptr(), _native.stream_ptr(dy2.device))
    return out


def _bgrad(dy2, b):
    if b is None:
        return None
    if has_main_grad(b) and _colsum_ok(dy2, b.main_grad):
        colsum_(dy2, b.main_grad, accumulate=main_grad_beta(b) != 0.0)
        return None
    if dy2.is_cuda and b.dtype in (torch.bfloat16, torch.float32):
        g = torch.empty(b.shape, device=b.device, dtype=b.dtype)
        if _colsum_ok(dy2, g):
            return colsum_(dy2, g)
    g = dy2.sum(0, dtype=torch.float32)  # f32 accumulation without an f32 copy of dy
    if has_main_grad(b):
        if main_grad_beta(b) == 0.0:
            b.main_grad.copy_(g.to(b.main_grad.dtype))
        else:
            b.main_grad.add_(g.to(b.main_grad.dtype))
        return None
    return g.to(b.dtype)


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, residual):
        x2 = rows2d(x)
        r2 = rows2d(residual) if residual is not None else None
        y = gemm(x2, w, trans_b=True, bias=b, residual=r2)
        ctx.save_for_backward(x2, w, b)
        ctx.xshape = x.shape
        ctx.has_res = residual is not None
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w, b = ctx.saved_tensors
        dy2 = rows2d(dy)
        dx = gemm(dy2, w).view(ctx.xshape) if ctx.needs_input_grad[0] else None
        dw = _wgrad(dy2, x2, w) if ctx.needs_input_grad[1] else None
        db = _bgrad(dy2, b) if (b is not None and ctx.needs_input_grad[2]) else None
        dres = dy if ctx.has_res else None
        return dx, dw, db, dres


def linear(x, w, b=None, residual=None):
    """y = x @ w.T (+ b) (+ residual)."""
    if x.is_cuda:
        return _LinearFn.apply(x, w, b, residual)
    y = torch.nn.functional.linear(x.float(), w.float(), None if b is None else b.float())
    if residual is not None:
        y = y + residual.float()
    return y.to(x.dtype)


class _NormLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, nw, w, eps, rope):
        x2 = rows2d(x)
        xn, _, _, rstd = _norms._fwd(_norms._RMS, x2, nw, None, eps)
        y = None
        if rope is not None:  # (table, heads rotated, head_dim, seq_len, offset)
            table, rot_heads, hd, S, off = rope
            y = gemm_rope(xn, w, table, rot_heads * hd, hd, S, off)
            if y is None:  # shapes outside the fused epilogue: rotate the q and k columns separately
                y = gemm(xn, w, trans_b=True)
                apply_rope_(y.view(-1, S, w.shape[0] // hd, hd)[:, :, :rot_heads], table, None, off)
        else:
            y = gemm(xn, w, trans_b=True)
        ctx.save_for_backward(x2, nw, w, rstd, rope[0] if rope is not None else torch.empty(0))
        ctx.rope = None if rope is None else rope[1:]
        ctx.eps = eps
        ctx.xshape = x.shape
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, nw, w, rstd, table = ctx.saved_tensors
        dy2 = rows2d(dy)
        if ctx.rope is not None:
            # gradient w.r.t. the unrotated projection: the inverse rotation of its q and k columns, on a
            # copy (autograd may hand the caller's own gradient tensor to this backward, and rotating
            # that in place would change it for every other reader)
            rot_heads, hd, S, off = ctx.rope
            dy2 = dy2.clone(memory_format=torch.contiguous_format)
            apply_rope_(dy2.view(-1, S, w.shape[0] // hd, hd)[:, :, :rot_heads], table, None, off, inverse=True)
        xn, _, _, _ = _norms._fwd(_norms._RMS, x2, nw, None, ctx.eps)  # recompute
        dxn = gemm(dy2, w)
        dw = _wgrad(dy2, xn, w)
        del xn
        dx, dnw, _ = _norms._bwd(_norms._RMS, dxn, x2, nw, None, None, rstd)
        return dx.view(ctx.xshape), dnw, dw, None, None


def norm_linear(x, norm_w, w, eps=1e-6, rope=None):
    """rms_norm(x, norm_w) @ w.T with the normalised activations recomputed in backward.

    ``rope = (table, rot_heads, head_dim, seq_len, offset)``: NeoX RoPE on the first ``rot_heads``
    heads of the output (the q and k heads of a fused QKV projection [.., (Hq + 2 Hkv) * head_dim]),
    applied in the GEMM epilogue where the shapes allow; the backward returns the gradient of the
    unrotated projection."""
    if x.is_cuda:
        return _NormLinearFn.apply(x, norm_w, w, eps, rope)
    y = linear(_norms.rms_norm_ref(x, norm_w, eps), w)
    if rope is not None:
        from .rope import rope_ref
        table, rot_heads, hd, S, off = rope
        y4 = y.view(-1, S, w.shape[0] // hd, hd)
        y4 = torch.cat([rope_ref(y4[:, :, :rot_heads], table, None, off), y4[:, :, rot_heads:]], dim=2)
        y = y4.reshape(y.shape)
    return y


class _SwiGLULinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu, w, residual):
        g2 = rows2d(gu)
        a = swiglu_fwd_only(g2)
        r2 = rows2d(residual) if residual is not None else None
        y = gemm(a, w, trans_b=True, residual=r2)
        ctx.save_for_backward(g2, w)
        ctx.gshape = gu.shape
        ctx.has_res = residual is not None
        return y.view(*gu.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        g2, w = ctx.saved_tensors
        dy2 = rows2d(dy)
        a = swiglu_fwd_only(g2)  # recompute the activation
        dw = _wgrad(dy2, a, w)
        da = gemm(dy2, w, out=a)  # reuse the activation buffer for its gradient
        dgu = swiglu_bwd_only(da, g2)
        return dgu.view(ctx.gshape), dw, (dy if ctx.has_res else None)


def swiglu_linear(gu, w, residual=None):
    """swiglu(gu) @ w.T (+ residual), recomputing swiglu(gu) in backward."""
    if gu.is_cuda:
        return _SwiGLULinearFn.apply(gu, w, residual)
    from .activations import swiglu_ref
    return linear(swiglu_ref(gu), w, residual=residual)


_NOT_SUPPORTED = 801  # cudaErrorNotSupported: the fused GEMM does not apply to this shape


def _gelu_dual(x2, w1, b1):
    """(h, gelu(h)) with h = x2 @ w1.T (+ b1): one GEMM with two outputs when it applies."""
    M, K = x2.shape
    F = w1.shape[0]
    h = torch.empty(M, F, device=x2.device, dtype=torch.bfloat16)
    a = torch.empty_like(h)
    rc = _native.fn("brain_gemm_bf16_gelu_dual")(
        x2.data_ptr(), x2.stride(0), w1.data_ptr(), w1.stride(0), h.data_ptr(), h.stride(0), a.data_ptr(),
        a.stride(0), M, F, K, b1.data_ptr() if b1 is not None else None, _native.stream_ptr(x2.device))
    if rc == _NOT_SUPPORTED:
        from .activations import gelu
        h = gemm(x2, w1, trans_b=True, bias=b1)
        return h, gelu(h)
    if rc != 0:
        raise _native.NativeError(f"brain_gemm_bf16_gelu_dual failed with status {rc}")
    return h, a


def _gelu_grad(dy2, w2, h):
    """(dy2 @ w2) * gelu'(h): the second layer's data gradient through the activation, one GEMM when it applies."""
    M, D = dy2.shape
    F = w2.shape[1]
    dh = torch.empty(M, F, device=dy2.device, dtype=torch.bfloat16)
    rc = _native.fn("brain_gemm_bf16_gelu_grad")(
        dy2.data_ptr(), dy2.stride(0), w2.data_ptr(), w2.stride(0), 1, dh.data_ptr(), dh.stride(0), h.data_ptr(),
        h.stride(0), M, F, D, _native.stream_ptr(dy2.device))
    if rc == _NOT_SUPPORTED:
        da = gemm(dy2, w2)
        _native.call("brain_gelu_bwd", da.data_ptr(), h.data_ptr(), dh.data_ptr(), dh.numel(),
                     _native.stream_ptr(dy2.device))
        return dh
    if rc != 0:
        raise _native.NativeError(f"brain_gemm_bf16_gelu_grad failed with status {rc}")
    return dh


class _GeluMLPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, residual):
        x2 = rows2d(x)
        h, a = _gelu_dual(x2, w1, b1)
        r2 = rows2d(residual) if residual is not None else None
        y = gemm(a, w2, trans_b=True, bias=b2, residual=r2)
        ctx.save_for_backward(x2, w1, b1, h, a, w2, b2)
        ctx.xshape = x.shape
        ctx.has_res = residual is not None
        return y.view(*x.shape[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w1, b1, h, a, w2, b2 = ctx.saved_tensors
        dy2 = rows2d(dy).contiguous()
        nig = ctx.needs_input_grad
        dw2 = _wgrad(dy2, a, w2) if nig[3] else None
        db2 = _bgrad(dy2, b2) if (b2 is not None and nig[4]) else None
        dh = _gelu_grad(dy2, w2, h)
        dx = gemm(dh, w1).view(ctx.xshape) if nig[0] else None
        dw1 = _wgrad(dh, x2, w1) if nig[1] else None
        db1 = _bgrad(dh, b1) if (b1 is not None and nig[2]) else None
        return dx, dw1, db1, dw2, db2, (dy if ctx.has_res else None)


def gelu_mlp(x, w1, b1, w2, b2, residual=None):
    """gelu(x @ w1.T + b1) @ w2.T + b2 (+ residual) with tanh GELU (the plain transformer MLP). On CUDA the
    first GEMM also writes gelu of its output (two TMA stores per tile), and the second layer's data
    gradient applies gelu' in its epilogue, so the activation costs no separate pass either way."""
    if x.is_cuda and x.dtype == torch.bfloat16:
        return _GeluMLPFn.apply(x, w1, b1, w2, b2, residual)
    from .activations import gelu
    return linear(gelu(linear(x, w1, b1)), w2, b2, residual)
