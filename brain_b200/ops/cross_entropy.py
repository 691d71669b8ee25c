"""Softmax cross-entropy (``csrc/cross_entropy.cu``) and the fused LM-head + cross-entropy op.

``cross_entropy(logits, labels, ignore_index, label_smoothing, reduction)`` matches the reference
CrossEntropyLoss (crates/brain-loss/src/classification/ce.rs:16-135; max-subtracted softmax,
crates/brain-core/src/tensor/special.rs:119-125) with mean over non-ignored rows.

``linear_cross_entropy(h, w, labels)`` is the LM head: it computes the logits with the tcgen05
GEMM, runs the loss forward, and immediately turns the logits buffer into d(loss)/d(logits) in
place (the upstream gradient of a scalar loss is folded into the backward GEMMs' alpha). Peak
memory is one [tokens, vocab] bf16 buffer, optionally processed in row chunks.
"""
from __future__ import annotations

import torch

from .. import _native
from ._common import has_main_grad, main_grad_beta, ptr, rows2d, stream
from .gemm import gemm


def _ce_fwd(logits2, labels, ignore_index, smoothing):
    M, V = logits2.shape
    loss = torch.empty(M, device=logits2.device, dtype=torch.float32)
    lse = torch.empty(M, device=logits2.device, dtype=torch.float32)
    _native.call("brain_ce_fwd", logits2.data_ptr(), logits2.stride(0), labels.data_ptr(), loss.data_ptr(),
                 lse.data_ptr(), M, V, int(ignore_index), float(smoothing), stream(logits2))
    return loss, lse


def _ce_bwd(logits2, labels, lse, grad_rows, grad_scalar, scale, out, ignore_index, smoothing):
    M, V = logits2.shape
    _native.call("brain_ce_bwd", logits2.data_ptr(), logits2.stride(0), labels.data_ptr(), lse.data_ptr(),
                 ptr(grad_rows), ptr(grad_scalar), float(scale), out.data_ptr(), out.stride(0), M, V,
                 int(ignore_index), float(smoothing), stream(logits2))
    return out


class _CEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, ignore_index, smoothing, reduction):
        l2 = rows2d(logits)
        lab = labels.reshape(-1).contiguous()
        loss, lse = _ce_fwd(l2, lab, ignore_index, smoothing)
        ctx.save_for_backward(l2, lab, lse)
        ctx.meta = (ignore_index, smoothing, reduction, logits.shape)
        if reduction == "none":
            return loss.view(labels.shape)
        n = (lab != ignore_index).sum().clamp_min(1) if reduction == "mean" else None
        ctx.n = n
        return loss.sum() / n if reduction == "mean" else loss.sum()

    @staticmethod
    def backward(ctx, g):
        l2, lab, lse = ctx.saved_tensors
        ignore_index, smoothing, reduction, shape = ctx.meta
        out = torch.empty_like(l2)
        if reduction == "none":
            _ce_bwd(l2, lab, lse, g.reshape(-1).float().contiguous(), None, 1.0, out, ignore_index, smoothing)
        else:
            gs = g.reshape(1).float()
            if reduction == "mean":
                gs = gs / ctx.n.float()
            _ce_bwd(l2, lab, lse, None, gs.contiguous(), 1.0, out, ignore_index, smoothing)
        return out.view(shape), None, None, None, None


def cross_entropy_ref(logits, labels, ignore_index=-100, label_smoothing=0.0, reduction="mean"):
    return torch.nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), labels.reshape(-1).long(),
                                             ignore_index=ignore_index, label_smoothing=label_smoothing,
                                             reduction=reduction)


def cross_entropy(logits, labels, ignore_index: int = -100, label_smoothing: float = 0.0, reduction: str = "mean"):
    if logits.is_cuda and logits.dtype == torch.bfloat16 and logits.shape[-1] % 8 == 0:
        return _CEFn.apply(logits, labels.long(), ignore_index, label_smoothing, reduction)
    return cross_entropy_ref(logits, labels, ignore_index, label_smoothing, reduction)


class _LinearCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, labels, ignore_index, smoothing, chunk):
        h2 = rows2d(h)
        lab = labels.reshape(-1).contiguous()
        M = h2.shape[0]
        V = w.shape[0]
        n = (lab != ignore_index).sum().clamp_min(1).float()
        inv_n = (1.0 / n).reshape(1)
        chunk = M if not chunk else min(chunk, M)
        total = torch.zeros((), device=h.device, dtype=torch.float32)
        dlogits = torch.empty(M, V, device=h.device, dtype=torch.bfloat16)
        for s0 in range(0, M, chunk):
            s1 = min(M, s0 + chunk)
            lg = dlogits[s0:s1]
            gemm(h2[s0:s1], w, trans_b=True, out=lg)
            loss, lse = _ce_fwd(lg, lab[s0:s1], ignore_index, smoothing)
            total += loss.sum()
            _ce_bwd(lg, lab[s0:s1], lse, None, inv_n, 1.0, lg, ignore_index, smoothing)  # in place
        ctx.save_for_backward(h2, w, dlogits)
        ctx.hshape = h.shape
        return total / n

    @staticmethod
    def backward(ctx, g):
        h2, w, dlogits = ctx.saved_tensors
        alpha = float(g)  # scalar loss: fold the upstream gradient into the GEMM alpha
        dh = gemm(dlogits, w, alpha=alpha)
        if has_main_grad(w):
            gemm(dlogits, h2, trans_a=True, out=w.main_grad, beta=main_grad_beta(w), alpha=alpha)
            dw = None
        else:
            dw = gemm(dlogits, h2, trans_a=True, out_dtype=torch.float32, alpha=alpha).to(w.dtype)
        return dh.view(ctx.hshape), dw, None, None, None, None


def linear_cross_entropy(h, w, labels, ignore_index: int = -100, label_smoothing: float = 0.0, chunk: int = 0):
    """mean CE of (h @ w.T) against labels, with the logits never materialised twice."""
    if h.is_cuda:
        return _LinearCEFn.apply(h, w, labels.long(), ignore_index, label_smoothing, chunk)
    logits = torch.nn.functional.linear(h.float(), w.float())
    return cross_entropy_ref(logits, labels, ignore_index, label_smoothing)
