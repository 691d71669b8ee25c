"""Embedding gather / deterministic scatter-add (``csrc/elementwise.cu``).

Forward gathers rows (plus an optional learned position table, as GPT-lite's embedding layer
does: crates/brain-transformer/src/embedding_layers.rs:153). Backward sorts the token ids once and
sums each id's rows in one CTA (no atomics, bit-reproducible), accumulating into ``main_grad``
when present (reference scatter-add VJP: crates/brain-autograd/src/ops/index_grad.rs:8).
"""
from __future__ import annotations

import torch

from .. import _native
from ._common import has_main_grad, main_grad_beta, ptr, stream


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w, pos):
        shape = ids.shape
        ids1 = ids.reshape(-1).contiguous().long()
        M = ids1.numel()
        V, D = w.shape
        S = shape[-1] if len(shape) > 1 else M
        out = torch.empty(M, D, device=w.device, dtype=w.dtype)
        _native.call("brain_embedding_fwd", ids1.data_ptr(), w.data_ptr(), ptr(pos), S, out.data_ptr(), M, D, V,
                     stream(w))
        ctx.save_for_backward(ids1, w, pos) if pos is not None else ctx.save_for_backward(ids1, w)
        ctx.meta = (S, pos is not None)
        return out.view(*shape, D)

    @staticmethod
    def backward(ctx, dy):
        S, has_pos = ctx.meta
        if has_pos:
            ids1, w, pos = ctx.saved_tensors
        else:
            ids1, w = ctx.saved_tensors
            pos = None
        V, D = w.shape
        dy2 = dy.reshape(-1, D).contiguous()
        M = dy2.shape[0]
        sorted_ids, perm = torch.sort(ids1)
        if has_main_grad(w):
            dw, ret = w.main_grad, None
            if main_grad_beta(w) == 0.0:  # sparse rows are accumulated: clear the first time
                dw.zero_()
        else:
            dw = torch.zeros(V, D, device=w.device, dtype=torch.float32)
            ret = dw
        _native.call("brain_embedding_bwd", sorted_ids.data_ptr(), perm.data_ptr(), dy2.data_ptr(), dw.data_ptr(),
                     int(dw.dtype == torch.float32), M, D, V, stream(dy))
        dpos = None
        if pos is not None:
            if has_main_grad(pos):
                dp = pos.main_grad
                if main_grad_beta(pos) == 0.0:
                    dp.zero_()
            else:
                dp = torch.zeros(pos.shape, device=pos.device, dtype=torch.float32)
                dpos = dp
            _native.call("brain_pos_grad", dy2.data_ptr(), dp.data_ptr(), int(dp.dtype == torch.float32), M, S, D,
                         stream(dy))
            if dpos is not None:
                dpos = dpos.to(pos.dtype)
        return None, (ret.to(w.dtype) if ret is not None else None), dpos


def embedding(ids: torch.Tensor, weight: torch.Tensor, pos_weight: torch.Tensor | None = None) -> torch.Tensor:
    """weight[ids] (+ pos_weight[position]) where position is the index along the last ids dim."""
    if weight.is_cuda and weight.dtype == torch.bfloat16 and weight.shape[1] % 8 == 0:
        return _EmbeddingFn.apply(ids, weight, pos_weight)
    out = torch.nn.functional.embedding(ids.long(), weight)
    if pos_weight is not None:
        S = ids.shape[-1]
        out = out + pos_weight[:S]
    return out
