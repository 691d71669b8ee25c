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


# ------------------------------------------------------------------ encoder side, rotary and positional encodings
# Reference: crates/brain-transformer/src/encoder/{mod,layer,block}.rs, position/rope.rs:15-200,
# position/mod.rs (PositionalEncoding: learned / sinusoidal), attention/multi_head.rs (split/merge heads),
# builder.rs (build_encoder / build_decoder).

class TransformerEncoderLayer(TransformerBlock):
    """Bidirectional self-attention + feed-forward (pre- or post-norm)."""

    def __init__(self, dim, heads, ffn_dim, **kw):
        kw.setdefault("causal", False)
        super().__init__(dim, heads, ffn_dim, **kw)


EncoderLayer = TransformerEncoderLayer
TransformerEncoderBlock = TransformerEncoderLayer


class TransformerEncoder(Module):
    def __init__(self, num_layers, dim, heads, ffn_dim, final_norm: bool = True, **kw):
        super().__init__()
        self.layers = torch.nn.ModuleList([TransformerEncoderLayer(dim, heads, ffn_dim, **kw)
                                           for _ in range(num_layers)])
        self.norm = make_norm(kw.get("norm", "layer"), dim, kw.get("eps", 1e-5), kw.get("device"),
                              kw.get("dtype")) if final_norm else None

    def forward(self, x, mask=None, attn_bias=None):
        for layer in self.layers:
            x = layer(x, mask=mask, attn_bias=attn_bias)
        return self.norm(x) if self.norm is not None else x


def build_encoder(num_layers, dim, heads, ffn_dim, **kw) -> TransformerEncoder:
    return TransformerEncoder(num_layers, dim, heads, ffn_dim, **kw)


def build_decoder(num_layers, dim, heads, ffn_dim, **kw) -> TransformerDecoder:
    return TransformerDecoder(num_layers, dim, heads, ffn_dim, **kw)


@dataclass
class RopeConfig:
    dim: int = 64
    max_seq_len: int = 2048
    theta: float = 10000.0
    scaling_factor: float = 1.0
    is_2d: bool = False


class RotaryEmbedding:
    """Rotary position embedding with the half-split pairing (x_i, x_{i + D/2}) and angle
    (pos / scaling_factor) theta^(-2i/D). The float32 cos/sin table lives on the device; ``apply_rope_4d``
    rotates [B, H, S, D] in place with the rope kernel on CUDA (positions at or past max_seq_len are left
    unrotated, as in the reference)."""

    def __init__(self, config: RopeConfig | None = None, device=None):
        from ..ops.rope import rope_table
        self.config = c = config or RopeConfig()
        self.table = rope_table(c.dim, c.max_seq_len, c.theta, device or "cpu", 1.0 / c.scaling_factor)

    @staticmethod
    def compute_frequencies(dim, max_seq_len, theta, scaling_factor=1.0):
        """(cos, sin), each float64 [max_seq_len, dim / 2]."""
        th = float(torch.tensor(theta, dtype=torch.float32))
        freq = 1.0 / th ** (torch.arange(dim // 2, dtype=torch.float64) * 2 / dim)
        ang = (torch.arange(max_seq_len, dtype=torch.float64) / scaling_factor)[:, None] * freq[None]
        return ang.cos(), ang.sin()

    def _table_for(self, x):
        if self.table.device != x.device:
            self.table = self.table.to(x.device)
        return self.table

    def apply_rope_4d(self, x: torch.Tensor, pos_offset: int = 0) -> torch.Tensor:
        from ..ops.rope import apply_rope_
        if x.dim() != 4:
            raise ValueError(f"apply_rope_4d expects [B, H, S, D], got {tuple(x.shape)}")
        n = max(0, min(x.shape[2], self.config.max_seq_len - pos_offset))
        if n:
            apply_rope_(x[:, :, :n].transpose(1, 2), self._table_for(x), offset=pos_offset)
        return x

    def apply_rope_2d(self, x: torch.Tensor, height: int, width: int) -> torch.Tensor:
        """[B, H, height*width, D] patches: quarter 1/2 of D rotate with the row, quarter 3/4 with the
        column, each with the table's first D/4 frequencies."""
        B, H, N, D = x.shape
        if N != height * width:
            raise ValueError(f"{N} patches != {height} x {width}")
        q = D // 4
        t = self._table_for(x)
        half = self.config.dim // 2
        cos, sin = t[:, :half][:, :q], t[:, half:][:, :q]
        rows = torch.arange(height, device=x.device).repeat_interleave(width)
        cols = torch.arange(width, device=x.device).repeat(height)
        xf = x.float()
        out = xf.clone()
        for base, idx in ((0, rows), (2 * q, cols)):
            c, s = cos[idx], sin[idx]
            a, b = xf[..., base:base + q], xf[..., base + q:base + 2 * q]
            out[..., base:base + q] = a * c - b * s
            out[..., base + q:base + 2 * q] = a * s + b * c
        x.copy_(out.to(x.dtype))
        return x


class PositionalEncoding(Module):
    """Absolute positions added to token embeddings [B, S, D]: ``kind`` "sinusoidal" (fixed table) or
    "learned" (a trained [max_len, D] table)."""

    def __init__(self, dim: int, max_len: int = 2048, kind: str = "sinusoidal", device=None, dtype=None):
        super().__init__()
        from .position import sinusoidal
        self.kind = kind
        if kind == "sinusoidal":
            self.register_buffer("pe", sinusoidal(max_len, dim).to(device=device, dtype=dtype or torch.float32))
        elif kind == "learned":
            self.pe = torch.nn.Parameter(torch.randn(max_len, dim, device=device, dtype=dtype or torch.float32) * 0.02)
        else:
            raise ValueError(f"unknown positional encoding {kind!r}")

    def forward(self, x, offset: int = 0):
        return x + self.pe[offset:offset + x.shape[1]].to(x.dtype)


class RelativePositionBias(RelativeAttention):
    """The T5 bucketed bias on its own: ``compute_bias(sq, sk)`` -> [H, sq, sk]."""

    def compute_bias(self, sq: int, sk: int) -> torch.Tensor:
        return self.bias(sq, sk)


def split_heads(x: torch.Tensor, num_heads: int) -> torch.Tensor:
    """[B, S, H*D] -> [B, H, S, D]."""
    B, S, E = x.shape
    return x.view(B, S, num_heads, E // num_heads).transpose(1, 2)


def merge_heads(x: torch.Tensor) -> torch.Tensor:
    """[B, H, S, D] -> [B, S, H*D]."""
    B, H, S, D = x.shape
    return x.transpose(1, 2).reshape(B, S, H * D)
