"""Position encodings (crates/brain-transformer/src/position/*.rs): sinusoidal (learned.rs:36-110
``SinusoidalPositionalEmbedding::generate``), learned tables, ALiBi slopes and biases
(alibi.rs:49-120), RoPE tables with a position scale factor (rope.rs:57-78) and the 2-D RoPE used for
image patches (rope.rs:145-201)."""
from __future__ import annotations

import math

import torch

from ..ops.rope import rope_table


def sinusoidal(max_len: int, dim: int, base: float = 10000.0) -> torch.Tensor:
    """[max_len, dim] with sin on even and cos on odd feature indices."""
    pos = torch.arange(max_len, dtype=torch.float64)[:, None]
    i = torch.arange(0, dim, 2, dtype=torch.float64)
    ang = pos / base ** (i / dim)
    pe = torch.zeros(max_len, dim, dtype=torch.float64)
    pe[:, 0::2] = torch.sin(ang)
    pe[:, 1::2] = torch.cos(ang[:, : dim // 2])
    return pe.float()


def alibi_slopes(num_heads: int) -> torch.Tensor:
    """Geometric slopes 2^(-8 i / n) for a power of two n, interleaved extension otherwise."""
    def pow2(n):
        start = 2 ** (-(2 ** -(math.log2(n) - 3)))
        return [start * start ** i for i in range(n)]
    if math.log2(num_heads).is_integer():
        s = pow2(num_heads)
    else:
        c = 2 ** math.floor(math.log2(num_heads))
        s = pow2(c) + pow2(2 * c)[0::2][: num_heads - c]
    return torch.tensor(s, dtype=torch.float32)


def alibi_bias(num_heads: int, q_len: int, k_len: int, causal: bool = True, device=None) -> torch.Tensor:
    """Additive [H, q_len, k_len] bias -slope * distance (bottom-right aligned positions)."""
    slopes = alibi_slopes(num_heads).to(device)
    qpos = torch.arange(q_len, device=device)[:, None] + (k_len - q_len)
    kpos = torch.arange(k_len, device=device)[None, :]
    dist = (qpos - kpos).float()
    if not causal:
        dist = dist.abs()
    return -slopes[:, None, None] * dist[None]


def rope(dim: int, max_pos: int, theta: float = 10000.0, scale: float = 1.0, device="cpu") -> torch.Tensor:
    return rope_table(dim, max_pos, theta, device, scale)


def rope_2d(x: torch.Tensor, grid_h: int, grid_w: int, theta: float = 10000.0) -> torch.Tensor:
    """2-D rotary embedding for patch tokens [B, H*W, heads, D]: the first half of D rotates with the
    row index, the second half with the column index."""
    from ..ops.rope import rope_ref
    B, N, H, D = x.shape
    half = D // 2
    rows = torch.arange(grid_h).repeat_interleave(grid_w)[None].expand(B, N)
    cols = torch.arange(grid_w).repeat(grid_h)[None].expand(B, N)
    t = rope_table(half, max(grid_h, grid_w), theta)
    a = rope_ref(x[..., :half].float(), t, rows)
    b = rope_ref(x[..., half:].float(), t, cols)
    return torch.cat([a, b], -1).to(x.dtype)


class LearnedPositionalEmbedding(torch.nn.Module):
    def __init__(self, max_len: int, dim: int):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.zeros(max_len, dim))
        torch.nn.init.normal_(self.weight, std=0.02)

    def forward(self, seq_len: int, offset: int = 0):
        return self.weight[offset: offset + seq_len]
