"""The reference's remaining transformer entry points, as thin front-ends over this framework's kernels:
``FlashAttentionLite`` / ``XformersAttentionLite`` (tiled attention configurations), ``RelativeAttention``
(T5 bucketed bias), ``AlibiPositionalBias``, ``LayerKvCache`` (one layer's contiguous cache), an
encoder-decoder ``TransformerDecoderLayer`` / ``TransformerDecoder``, ``repeat_kv``, ``quick_gelu`` and
``all_close``.

Reference: crates/brain-transformer/src/attention/flash_lite.rs (FlashLiteConfig: block_m, block_n,
scale, is_causal), attention/xformers_lite.rs (XformersConfig: chunk_size), attention/relative.rs,
position/alibi.rs, kv_cache.rs (LayerKvCache), decoder/layer.rs (TransformerDecoderLayer: self-attention,
optional cross-attention, FFN), attention/multi_query.rs (repeat_kv), ops.rs (quick_gelu), utils
(all_close).

On CUDA bf16/f16 inputs without a bias the attention classes run the tcgen05 flash kernels (their block
sizes are the kernels' own: 128-row query tiles, 128-key blocks); with a bias, or on the CPU, they run
the tiled online-softmax path with the configured block / chunk sizes. Causal masks are bottom-right
aligned, so decode steps (fewer queries than keys) attend to the whole prefix.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..nn.module import Module
from ..ops import attention as attn
from .blocks import TransformerBlock, make_norm, memory_efficient_attention
from .families import relative_position_bucket
from .position import alibi_slopes


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """[B, H_kv, S, D] -> [B, H_kv n_rep, S, D], each key/value head repeated for its query group."""
    if n_rep == 1:
        return x
    if x.dim() != 4:
        raise ValueError(f"repeat_kv expects [B, H, S, D], got {tuple(x.shape)}")
    B, H, S, D = x.shape
    return x[:, :, None].expand(B, H, n_rep, S, D).reshape(B, H * n_rep, S, D)


def quick_gelu(x: torch.Tensor) -> torch.Tensor:
    """x sigmoid(1.702 x)."""
    return x * torch.sigmoid(1.702 * x)


def all_close(a: torch.Tensor, b: torch.Tensor, rtol: float = 1e-5, atol: float = 1e-8) -> bool:
    return a.shape == b.shape and bool(torch.allclose(a.double(), b.double(), rtol=rtol, atol=atol))


@dataclass
class FlashLiteConfig:
    block_m: int = 64
    block_n: int = 64
    scale: float | None = None
    is_causal: bool = False


@dataclass
class XformersConfig:
    chunk_size: int = 64
    scale: float | None = None
    is_causal: bool = False


def _fast_ok(q, bias):
    return bias is None and q.is_cuda and q.dtype in (torch.bfloat16, torch.float16)


class FlashAttentionLite:
    """attention(q, k, v [B, S, H, D], bias=None): the tcgen05 flash kernels on GPU, else query/key
    tiles of block_m x block_n with an online softmax."""

    def __init__(self, config: FlashLiteConfig | None = None):
        self.c = config or FlashLiteConfig()

    def forward(self, q, k, v, bias=None):
        D = q.shape[-1]
        scale = self.c.scale
        if _fast_ok(q, bias):
            return attn.flash_attention(q, k, v, causal=self.c.is_causal, scale=scale)
        if scale is not None:
            q = q * (scale * math.sqrt(D))
        return memory_efficient_attention(q, k, v, bias, self.c.is_causal, self.c.block_m, self.c.block_n).to(q.dtype)

    __call__ = forward


class XformersAttentionLite(FlashAttentionLite):
    """Memory-efficient attention with square chunks of ``chunk_size`` queries and keys."""

    def __init__(self, config: XformersConfig | None = None):
        c = config or XformersConfig()
        super().__init__(FlashLiteConfig(c.chunk_size, c.chunk_size, c.scale, c.is_causal))


class AlibiPositionalBias:
    """ALiBi: per-head slopes (geometric, 2^(-8 i / H)) times the key-minus-query distance."""

    def __init__(self, num_heads: int):
        self.num_heads = num_heads
        self.slopes = alibi_slopes(num_heads)

    def bias(self, sq: int, sk: int, causal: bool = True, device=None):
        return attn.alibi_relative_bias(self.num_heads, sq, sk, causal=causal, device=device)


class RelativeAttention(Module):
    """Self-attention with a learned T5 relative-position bias (bucketed distances, one scalar per
    bucket and head) over [B, S, H, D] projections supplied by the caller."""

    def __init__(self, num_heads: int, num_buckets: int = 32, max_distance: int = 128, bidirectional: bool = True,
                 device=None, dtype=None):
        super().__init__()
        self.h, self.nb, self.md, self.bi = num_heads, num_buckets, max_distance, bidirectional
        self.table = torch.nn.Parameter(torch.zeros(num_buckets, num_heads, device=device,
                                                    dtype=dtype or torch.float32))

    def bias(self, sq: int, sk: int) -> torch.Tensor:
        """[H, sq, sk] additive bias (rows: queries aligned to the end of the keys)."""
        qp = torch.arange(sq, device=self.table.device)[:, None] + (sk - sq)
        kp = torch.arange(sk, device=self.table.device)[None, :]
        b = relative_position_bucket(kp - qp, self.bi, self.nb, self.md)
        return self.table[b].permute(2, 0, 1)

    def forward(self, q, k, v, causal: bool = False, key_mask=None):
        bias = self.bias(q.shape[1], k.shape[1])
        return attn.masked_attention(q, k, v, causal, key_mask, bias)


class LayerKvCache:
    """One layer's contiguous K/V cache [B, H_kv, max_len, D] with an append cursor."""

    def __init__(self, batch_size: int, num_kv_heads: int, head_dim: int, max_seq_len: int, device=None,
                 dtype=torch.bfloat16):
        self.k = torch.zeros(batch_size, num_kv_heads, max_seq_len, head_dim, device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.current_seq_len, self.max_seq_len = 0, max_seq_len

    def update(self, k: torch.Tensor, v: torch.Tensor):
        """Append [B, H_kv, S_new, D] and return views of the whole cached prefix."""
        n = k.shape[2]
        if self.current_seq_len + n > self.max_seq_len:
            raise ValueError(f"cache full: {self.current_seq_len} + {n} > {self.max_seq_len}")
        s = self.current_seq_len
        self.k[:, :, s:s + n] = k
        self.v[:, :, s:s + n] = v
        self.current_seq_len += n
        return self.k[:, :, :self.current_seq_len], self.v[:, :, :self.current_seq_len]

    def clear(self) -> None:
        self.current_seq_len = 0


class TransformerDecoderLayer(TransformerBlock):
    """Causal self-attention, cross-attention to an encoder memory, feed-forward (pre- or post-norm)."""

    def __init__(self, dim, heads, ffn_dim, cross: bool = True, **kw):
        kw.setdefault("causal", True)
        super().__init__(dim, heads, ffn_dim, cross=cross, **kw)


class TransformerDecoder(Module):
    def __init__(self, num_layers, dim, heads, ffn_dim, final_norm: bool = True, **kw):
        super().__init__()
        self.layers = torch.nn.ModuleList([TransformerDecoderLayer(dim, heads, ffn_dim, **kw)
                                           for _ in range(num_layers)])
        self.norm = make_norm(kw.get("norm", "layer"), dim, kw.get("eps", 1e-5), kw.get("device"),
                              kw.get("dtype")) if final_norm else None

    def forward(self, x, memory=None, mem_mask=None):
        for layer in self.layers:
            x = layer(x, mem=memory, mem_mask=mem_mask)
        return self.norm(x) if self.norm is not None else x
