"""Configurable transformer blocks shared by the GPT / BERT / T5 / ViT families.

Mirrors the reference's encoder/decoder stacks (crates/brain-transformer/src/encoder/*.rs,
decoder/mod.rs:60-150, decoder/layer.rs:60-260): pre- or post-norm, LayerNorm or RMSNorm, GELU
(tanh) or SwiGLU FFN, optional causal self-attention and cross-attention, and a final norm.
Self-attention runs the flash kernels through a fused QKV projection; key padding masks and relative
biases (ALiBi, T5 buckets without a gradient) run on the masked tcgen05 kernels
(``ops.attention.masked_attention``), a learned bias that needs its gradient on the float32 reference SDPA.
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..nn.layers import FeedForward, LayerNorm, Linear, RMSNorm
from ..nn.module import Module, ModuleList


def make_norm(kind: str, dim: int, eps: float, device=None, dtype=None):
    return RMSNorm(dim, eps, device, dtype) if kind == "rms" else LayerNorm(dim, eps, True, device, dtype)


def sdpa_with_bias(q, k, v, bias=None, causal=False, mask=None, scale=None):
    """[B, S, H, D] attention with an additive [H, Sq, Sk] / [B, H, Sq, Sk] bias (float32)."""
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qf, kf, vf = (x.float().transpose(1, 2) for x in (q, k, v))
    if kf.shape[1] != qf.shape[1]:
        rep = qf.shape[1] // kf.shape[1]
        kf, vf = kf.repeat_interleave(rep, 1), vf.repeat_interleave(rep, 1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if bias is not None:
        s = s + bias.float()
    Sq, Sk = s.shape[-2], s.shape[-1]
    if causal:
        i = torch.arange(Sq, device=q.device)[:, None]
        j = torch.arange(Sk, device=q.device)[None, :]
        s = s.masked_fill(j > i + (Sk - Sq), float("-inf"))
    if mask is not None:  # [B, Sk] padding mask, True = keep
        s = s.masked_fill(~mask[:, None, None, :].bool(), float("-inf"))
    p = torch.nan_to_num(torch.softmax(s, -1), nan=0.0)
    return (p @ vf).transpose(1, 2).to(q.dtype)


def memory_efficient_attention(q, k, v, bias=None, causal=False, q_chunk: int = 512, k_chunk: int = 512):
    """Tiled attention with an online softmax over key blocks (the reference's xformers-lite / flash-lite
    CPU tiling, crates/brain-transformer/src/attention/xformers_lite.rs and flash_lite.rs:46-222): memory
    O(q_chunk * k_chunk) per head instead of O(Sq * Sk), with the same optional additive bias
    ([H, Sq, Sk] or [B, H, Sq, Sk], sliced per tile) and bottom-right causal alignment as
    ``sdpa_with_bias``. For biased attention (ALiBi, T5 relative) at lengths where the full score matrix
    does not fit; unbiased attention uses the tcgen05 flash kernels."""
    B, Sq, H, D = q.shape
    Sk = k.shape[1]
    rep = H // k.shape[2]
    qf = q.float().transpose(1, 2) / math.sqrt(D)
    kf, vf = k.float().transpose(1, 2), v.float().transpose(1, 2)
    if rep > 1:
        kf, vf = kf.repeat_interleave(rep, 1), vf.repeat_interleave(rep, 1)
    out = torch.empty_like(qf)
    for q0 in range(0, Sq, q_chunk):
        q1 = min(Sq, q0 + q_chunk)
        m = torch.full((B, H, q1 - q0, 1), float("-inf"), device=q.device)
        l = torch.zeros((B, H, q1 - q0, 1), device=q.device)
        acc = torch.zeros((B, H, q1 - q0, D), device=q.device)
        for k0 in range(0, Sk, k_chunk):
            k1 = min(Sk, k0 + k_chunk)
            if causal and k0 > q1 - 1 + (Sk - Sq):
                break
            s = qf[:, :, q0:q1] @ kf[:, :, k0:k1].transpose(-1, -2)
            if bias is not None:
                s = s + bias[..., q0:q1, k0:k1].float()
            if causal:
                i = torch.arange(q0, q1, device=q.device)[:, None]
                j = torch.arange(k0, k1, device=q.device)[None, :]
                s = s.masked_fill(j > i + (Sk - Sq), float("-inf"))
            m_new = torch.maximum(m, s.amax(-1, keepdim=True))
            safe = torch.where(torch.isinf(m_new), torch.zeros_like(m_new), m_new)
            p = torch.exp(s - safe)
            corr = torch.exp(torch.where(torch.isinf(m), torch.full_like(m, float("-inf")), m - safe))
            l = l * corr + p.sum(-1, keepdim=True)
            acc = acc * corr + p @ vf[:, :, k0:k1]
            m = m_new
        out[:, :, q0:q1] = acc / l.clamp_min(1e-30)
    return out.transpose(1, 2).to(q.dtype)


class SelfAttention(Module):
    def __init__(self, dim, heads, kv_heads=None, bias=False, causal=False, device=None, dtype=None):
        super().__init__()
        self.h, self.hkv = heads, kv_heads or heads
        self.hd = dim // heads
        self.causal = causal
        self.qkv = Linear(dim, (self.h + 2 * self.hkv) * self.hd, bias=bias, device=device, dtype=dtype)
        self.out = Linear(self.h * self.hd, dim, bias=bias, device=device, dtype=dtype)

    def forward(self, x, residual=None, rope=None, attn_bias=None, mask=None):
        qkv = self.qkv(x)
        if attn_bias is None and mask is None:
            o = ops.qkv_attention(qkv, self.h, self.hkv, rope, causal=self.causal)
        else:
            # padding masks and relative biases (ALiBi, T5 buckets) on the tcgen05 kernels where possible
            q, k, v = ops.attention.split_qkv(qkv, self.h, self.hkv)
            o = ops.attention.masked_attention(q, k, v, self.causal, mask, attn_bias)
            o = o.reshape(x.shape[0], x.shape[1], -1)
        return self.out(o, residual)


class CrossAttention(Module):
    def __init__(self, dim, heads, bias=False, device=None, dtype=None):
        super().__init__()
        self.h, self.hd = heads, dim // heads
        self.q = Linear(dim, dim, bias=bias, device=device, dtype=dtype)
        self.kv = Linear(dim, 2 * dim, bias=bias, device=device, dtype=dtype)
        self.out = Linear(dim, dim, bias=bias, device=device, dtype=dtype)

    def forward(self, x, mem, residual=None, mem_mask=None):
        B, S, _ = x.shape
        q = self.q(x).view(B, S, self.h, self.hd)
        kv = self.kv(mem).view(B, mem.shape[1], 2, self.h, self.hd)
        k, v = kv[:, :, 0], kv[:, :, 1]
        if mem_mask is None and x.is_cuda:
            o = ops.flash_attention(q, k, v, causal=False)
        else:
            o = ops.attention.masked_attention(q, k, v, False, mem_mask)
        return self.out(o.reshape(B, S, -1), residual)


class TransformerBlock(Module):
    def __init__(self, dim, heads, ffn_dim, *, kv_heads=None, norm="layer", act="gelu", pre_norm=True,
                 causal=False, cross=False, bias=False, eps=1e-5, device=None, dtype=None):
        super().__init__()
        self.pre_norm = pre_norm
        self.norm1 = make_norm(norm, dim, eps, device, dtype)
        self.attn = SelfAttention(dim, heads, kv_heads, bias, causal, device, dtype)
        self.cross = CrossAttention(dim, heads, bias, device, dtype) if cross else None
        self.norm_c = make_norm(norm, dim, eps, device, dtype) if cross else None
        self.norm2 = make_norm(norm, dim, eps, device, dtype)
        self.ffn = FeedForward(dim, ffn_dim, gated=(act == "swiglu"), bias=bias, device=device, dtype=dtype, act=act)

    def forward(self, x, rope=None, attn_bias=None, mask=None, mem=None, mem_mask=None):
        if self.pre_norm:
            x = self.attn(self.norm1(x), residual=x, rope=rope, attn_bias=attn_bias, mask=mask)
            if self.cross is not None:
                x = self.cross(self.norm_c(x), mem, residual=x, mem_mask=mem_mask)
            return self.ffn(self.norm2(x), residual=x)
        x = self.norm1(self.attn(x, residual=x, rope=rope, attn_bias=attn_bias, mask=mask))
        if self.cross is not None:
            x = self.norm_c(self.cross(x, mem, residual=x, mem_mask=mem_mask))
        return self.norm2(self.ffn(x, residual=x))


class TransformerStack(Module):
    def __init__(self, n, dim, heads, ffn_dim, final_norm=True, **kw):
        super().__init__()
        self.layers = ModuleList([TransformerBlock(dim, heads, ffn_dim, **kw) for _ in range(n)])
        norm, eps = kw.get("norm", "layer"), kw.get("eps", 1e-5)
        self.final = make_norm(norm, dim, eps, kw.get("device"), kw.get("dtype")) if final_norm else None

    def forward(self, x, **kw):
        for layer in self.layers:
            x = layer(x, **kw)
        return self.final(x) if self.final is not None else x
