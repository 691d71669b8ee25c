"""Flash attention front-ends (``csrc/attention.cu``).

* ``flash_attention(q, k, v, causal)`` on ``[B, S, H, D]`` tensors (any strides with unit stride on
  D; GQA when k/v have fewer heads), returning ``o [B, Sq, Hq, D]``.
* ``qkv_attention(qkv, Hq, Hkv, ...)`` consumes the fused projection ``[B, S, (Hq + 2 Hkv) * D]``:
  RoPE is applied in place on its q/k columns, attention reads q/k/v through strides, and the
  backward writes dq/dk/dv straight into one ``dqkv`` buffer before the inverse rotation. Nothing
  is copied or re-laid-out, and only qkv, o and the log-sum-exp are kept for the backward pass.

The CPU path is the reference SDPA (scale 1/sqrt(d), row-max-subtracted softmax) in float32 with
bottom-right-aligned causal masking.
"""
from __future__ import annotations

import math

import torch

from .. import _native
from ._common import i64_array, stream
from .rope import apply_rope_


def _strides3(t):
    return [t.stride(0), t.stride(1), t.stride(2)]


_NOT_SUPPORTED = 801  # cudaErrorNotSupported: layout outside the tensor-core kernel's domain
USE_TC = True  # tcgen05 forward when the layout allows; the mma.sync kernel otherwise


def _fwd(q, k, v, causal, scale, impl=None):
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    o = torch.empty(B, Sq, Hq, D, device=q.device, dtype=q.dtype)
    lse = torch.empty(B, Hq, Sq, device=q.device, dtype=torch.float32)
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), i64_array(_strides3(q) + _strides3(k) + _strides3(v)),
            o.data_ptr(), i64_array(_strides3(o)), lse.data_ptr(), B, Hq, Hkv, Sq, Sk, D, float(scale), int(causal),
            stream(q))
    use_tc = USE_TC if impl is None else impl == "tc"
    if use_tc:
        rc = _native.fn("brain_attn_fwd_tc")(*args)
        if rc == 0:
            return o, lse
        if rc != _NOT_SUPPORTED or impl == "tc":
            raise _native.NativeError(f"brain_attn_fwd_tc failed with status {rc}")
    _native.call("brain_attn_fwd", *args)
    return o, lse


def _bwd(q, k, v, o, lse, do, dq, dk, dv, causal, scale, impl=None):
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    delta = torch.empty(B * Hq * Sq, device=q.device, dtype=torch.float32)
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), i64_array(_strides3(q) + _strides3(k) + _strides3(v)),
            o.data_ptr(), i64_array(_strides3(o)), lse.data_ptr(), do.data_ptr(), i64_array(_strides3(do)),
            dq.data_ptr(), i64_array(_strides3(dq)), dk.data_ptr(), i64_array(_strides3(dk)), dv.data_ptr(),
            i64_array(_strides3(dv)), delta.data_ptr(), B, Hq, Hkv, Sq, Sk, D, float(scale), int(causal), stream(q))
    use_tc = USE_TC if impl is None else impl == "tc"
    if use_tc:
        rc = _native.fn("brain_attn_bwd_tc")(*args)
        if rc == 0:
            return
        if rc != _NOT_SUPPORTED or impl == "tc":
            raise _native.NativeError(f"brain_attn_bwd_tc failed with status {rc}")
    _native.call("brain_attn_bwd", *args)


def _check(t):
    if t.stride(3) != 1:
        raise ValueError("attention inputs need unit stride on the head dimension")


class _FlashFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        for t in (q, k, v):
            _check(t)
        o, lse = _fwd(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.scale = causal, scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        do = do if do.stride(3) == 1 else do.contiguous()
        dq = torch.empty_like(q, memory_format=torch.contiguous_format)
        dk = torch.empty(k.shape, device=k.device, dtype=k.dtype)
        dv = torch.empty(v.shape, device=v.device, dtype=v.dtype)
        _bwd(q, k, v, o, lse, do, dq, dk, dv, ctx.causal, ctx.scale)
        return dq, dk, dv, None, None


def sdpa_ref(q, k, v, causal=True, scale=None):
    """float32 reference SDPA on [B, S, H, D] with GQA and bottom-right causal alignment."""
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    rep = Hq // Hkv
    qf = q.float().transpose(1, 2)
    kf = k.float().transpose(1, 2).repeat_interleave(rep, dim=1)
    vf = v.float().transpose(1, 2).repeat_interleave(rep, dim=1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        i = torch.arange(Sq, device=q.device)[:, None]
        j = torch.arange(Sk, device=q.device)[None, :]
        s = s.masked_fill(j > i + (Sk - Sq), float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return (p @ vf).transpose(1, 2).to(q.dtype)


def flash_attention(q, k, v, causal: bool = True, scale: float | None = None):
    """Attention over [B, S, H, D] tensors; GQA when k/v have fewer heads than q."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if q.is_cuda:
        return _FlashFn.apply(q, k, v, causal, scale)
    return sdpa_ref(q, k, v, causal, scale)


def flash_attention_fwd(q, k, v, causal=True, scale=None):
    """Inference forward returning (o, lse) without autograd bookkeeping."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    return _fwd(q, k, v, causal, scale)


def split_qkv(qkv: torch.Tensor, Hq: int, Hkv: int):
    """Views q [B,S,Hq,D], k/v [B,S,Hkv,D] into a fused projection [B, S, (Hq+2Hkv)*D]."""
    B, S, W = qkv.shape
    D = W // (Hq + 2 * Hkv)
    x = qkv.view(B, S, Hq + 2 * Hkv, D)
    return x[:, :, :Hq], x[:, :, Hq:Hq + Hkv], x[:, :, Hq + Hkv:]


class _QKVAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, Hq, Hkv, table, causal, scale, offset):
        q, k, v = split_qkv(qkv, Hq, Hkv)
        if table is not None:
            apply_rope_(q, table, None, offset)
            apply_rope_(k, table, None, offset)
        o, lse = _fwd(q, k, v, causal, scale)
        ctx.save_for_backward(qkv, o, lse, table if table is not None else torch.empty(0))
        ctx.meta = (Hq, Hkv, causal, scale, offset, table is not None)
        B, S = qkv.shape[:2]
        return o.view(B, S, -1)

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse, table = ctx.saved_tensors
        Hq, Hkv, causal, scale, offset, has_rope = ctx.meta
        q, k, v = split_qkv(qkv, Hq, Hkv)
        B, S = qkv.shape[:2]
        do4 = do.reshape(B, S, Hq, -1)
        if do4.stride(3) != 1:
            do4 = do4.contiguous()
        dqkv = torch.empty_like(qkv)
        dq, dk, dv = split_qkv(dqkv, Hq, Hkv)
        _bwd(q, k, v, o, lse, do4, dq, dk, dv, causal, scale)
        if has_rope:
            apply_rope_(dq, table, None, offset, inverse=True)
            apply_rope_(dk, table, None, offset, inverse=True)
        return dqkv, None, None, None, None, None, None


def qkv_attention(qkv: torch.Tensor, Hq: int, Hkv: int, rope_table: torch.Tensor | None = None, causal: bool = True,
                  scale: float | None = None, offset: int = 0) -> torch.Tensor:
    """Attention on a fused projection qkv [B, S, (Hq+2Hkv)*D] -> [B, S, Hq*D] (RoPE optional).

    On CUDA the RoPE rotation is applied in place to ``qkv`` (the projection output is owned by
    this op); the CPU path is out of place.
    """
    D = qkv.shape[-1] // (Hq + 2 * Hkv)
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if qkv.is_cuda:
        return _QKVAttnFn.apply(qkv, Hq, Hkv, rope_table, causal, scale, offset)
    from .rope import rope_ref
    q, k, v = split_qkv(qkv, Hq, Hkv)
    if rope_table is not None:
        q = rope_ref(q, rope_table, None, offset)
        k = rope_ref(k, rope_table, None, offset)
    o = sdpa_ref(q, k, v, causal, scale)
    return o.reshape(qkv.shape[0], qkv.shape[1], -1)


# --------------------------------------------------------------------------- masks and relative biases
class RelativeBias:
    """An additive attention bias that depends only on the key-query offset: ``vec[h, (k - q) + Sq - 1]``
    (float32, natural-log units, ``[Hq, Sq + Sk - 1]``), as ALiBi and T5's relative buckets are. The
    tcgen05 kernels read the vector directly; ``dense()`` materialises ``[Hq, Sq, Sk]`` for the
    float32 reference path (differentiable when ``vec`` is)."""

    def __init__(self, vec: torch.Tensor, Sq: int, Sk: int):
        if vec.shape[-1] != Sq + Sk - 1:
            raise ValueError(f"relative bias length {vec.shape[-1]} != Sq + Sk - 1 = {Sq + Sk - 1}")
        self.vec, self.Sq, self.Sk = vec, Sq, Sk

    def dense(self) -> torch.Tensor:
        q = torch.arange(self.Sq, device=self.vec.device)[:, None]
        k = torch.arange(self.Sk, device=self.vec.device)[None, :]
        return self.vec[:, k - q + self.Sq - 1]


def alibi_relative_bias(num_heads: int, Sq: int, Sk: int, causal: bool = True, device=None) -> RelativeBias:
    """ALiBi (crates/brain-transformer/src/position/alibi.rs:49-120) as a relative bias: -slope_h times the
    distance between the bottom-right aligned query position q + Sk - Sq and key k (absolute distance
    when not causal); the same values as ``models.position.alibi_bias``."""
    from ..models.position import alibi_slopes
    d = torch.arange(-(Sq - 1), Sk, device=device, dtype=torch.float32) - (Sk - Sq)  # k - (q + Sk - Sq)
    dist = -d if causal else d.abs()
    return RelativeBias((-alibi_slopes(num_heads).to(device)[:, None] * dist[None]).contiguous(), Sq, Sk)


def _tc_ok(q, k, v):
    D = q.shape[-1]
    return (q.is_cuda and q.dtype == torch.bfloat16 and D in (64, 128)
            and all(t.stride(-1) == 1 and all((s * 2) % 16 == 0 for s in t.stride()[:-1]) for t in (q, k, v)))


class _MaskedFlashFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale, kmask, relb):
        B, Sq, Hq, D = q.shape
        Sk, Hkv = k.shape[1], k.shape[2]
        o = torch.empty(B, Sq, Hq, D, device=q.device, dtype=q.dtype)
        lse = torch.empty(B, Hq, Sq, device=q.device, dtype=torch.float32)
        _native.call("brain_attn_fwd_tc_masked", q.data_ptr(), k.data_ptr(), v.data_ptr(),
                     i64_array(_strides3(q) + _strides3(k) + _strides3(v)), o.data_ptr(), i64_array(_strides3(o)),
                     lse.data_ptr(), B, Hq, Hkv, Sq, Sk, D, float(scale), int(causal),
                     0 if kmask is None else kmask.data_ptr(), 0 if relb is None else relb.data_ptr(), stream(q))
        ctx.save_for_backward(q, k, v, o, lse, *(t for t in (kmask, relb) if t is not None))
        ctx.meta = (causal, scale, kmask is not None, relb is not None)
        return o

    @staticmethod
    def backward(ctx, do):
        causal, scale, has_m, has_b = ctx.meta
        q, k, v, o, lse, *rest = ctx.saved_tensors
        kmask = rest.pop(0) if has_m else None
        relb = rest.pop(0) if has_b else None
        do = do if do.stride(3) == 1 else do.contiguous()
        B, Sq, Hq, D = q.shape
        Sk, Hkv = k.shape[1], k.shape[2]
        dq = torch.empty_like(q, memory_format=torch.contiguous_format)
        dk = torch.empty(k.shape, device=k.device, dtype=k.dtype)
        dv = torch.empty(v.shape, device=v.device, dtype=v.dtype)
        delta = torch.empty(B * Hq * Sq, device=q.device, dtype=torch.float32)
        _native.call("brain_attn_bwd_tc_masked", q.data_ptr(), k.data_ptr(), v.data_ptr(),
                     i64_array(_strides3(q) + _strides3(k) + _strides3(v)), o.data_ptr(), i64_array(_strides3(o)),
                     lse.data_ptr(), do.data_ptr(), i64_array(_strides3(do)), dq.data_ptr(), i64_array(_strides3(dq)),
                     dk.data_ptr(), i64_array(_strides3(dk)), dv.data_ptr(), i64_array(_strides3(dv)), delta.data_ptr(),
                     B, Hq, Hkv, Sq, Sk, D, float(scale), int(causal), 0 if kmask is None else kmask.data_ptr(),
                     0 if relb is None else relb.data_ptr(), stream(q))
        return dq, dk, dv, None, None, None, None


def masked_attention(q, k, v, causal: bool = False, key_mask: torch.Tensor | None = None,
                     bias: "RelativeBias | torch.Tensor | None" = None, scale: float | None = None):
    """Attention on [B, S, H, D] (GQA allowed) with a key padding mask ``[B, Sk]`` (True = attend) and/or an
    additive bias: a :class:`RelativeBias` (ALiBi, T5 buckets) or a dense ``[H, Sq, Sk]`` /
    ``[B, H, Sq, Sk]`` tensor (crates/brain-transformer/src/core.rs:81-107 ``AttentionMask::{Padding,
    AdditiveBias, CausalWithPadding}``). The tcgen05 kernels run it when the inputs are bf16 CUDA tensors
    with head_dim 64 / 128 and the bias is a relative one that needs no gradient; otherwise the float32
    reference SDPA does, which also gives the gradient of a learned bias."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    rel = bias if isinstance(bias, RelativeBias) else None
    kernel = _tc_ok(q, k, v) and (bias is None or (rel is not None and not rel.vec.requires_grad))
    if kernel:
        km = None if key_mask is None else key_mask.to(device=q.device, dtype=torch.uint8).contiguous()
        rb = None if rel is None else rel.vec.detach().to(device=q.device, dtype=torch.float32).contiguous()
        return _MaskedFlashFn.apply(q, k, v, causal, scale, km, rb)
    dense = rel.dense() if rel is not None else bias
    from ..models.blocks import sdpa_with_bias
    return sdpa_with_bias(q, k, v, dense, causal, key_mask, scale=scale)
