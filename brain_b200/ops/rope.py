"""Rotary position embedding (NeoX half-split), ``csrc/elementwise.cu``.

Pairs are ``(x[i], x[i + d/2])`` with ``freq_i = theta^(-2i/d)`` and the angle ``pos * freq_i *
scale`` (crates/brain-transformer/src/position/rope.rs:57-142, including the position scaling
factor at :70). The cos/sin table is built once per (device, dim, theta, length) in float32
(computed in float64 then rounded) and shared by every layer.
"""
from __future__ import annotations

import torch

from .. import _native
from ._common import ptr, stream

_TABLES: dict = {}


def rope_table(dim: int, max_pos: int, theta: float = 10000.0, device="cpu", scale: float = 1.0) -> torch.Tensor:
    """float32 [max_pos, dim]: cos in [:, :dim/2], sin in [:, dim/2:]."""
    key = (str(device), dim, max_pos, float(theta), float(scale))
    t = _TABLES.get(key)
    if t is None:
        half = dim // 2
        # theta is stored as f32 in the reference config; keep the same rounding.
        th = float(torch.tensor(theta, dtype=torch.float32))
        inv = th ** (-torch.arange(half, dtype=torch.float64) * 2.0 / dim)
        ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * scale * inv[None, :]
        t = torch.cat([ang.cos(), ang.sin()], dim=1).to(torch.float32).to(device)
        _TABLES[key] = t
    return t


def apply_rope_(x: torch.Tensor, table: torch.Tensor, positions: torch.Tensor | None = None, offset: int = 0,
                inverse: bool = False) -> torch.Tensor:
    """Rotate x [B, S, H, D] in place (any strides, unit stride on D). Returns x. bf16 CUDA tensors go
    through the rope kernel; other dtypes are rotated with tensor ops on their device."""
    B, S, H, D = x.shape
    if x.is_cuda and x.dtype == torch.bfloat16:
        if x.stride(3) != 1:
            raise ValueError("rope needs unit stride on the head dimension")
        pos = positions.to(torch.int32).contiguous() if positions is not None else None
        if pos is None and offset + S > table.shape[0]:
            raise ValueError(f"rope table has {table.shape[0]} positions, need {offset + S}")
        if table.shape[1] != D or not table.is_cuda:
            raise ValueError("rope table must be a CUDA float32 [max_pos, head_dim] tensor")
        _native.call("brain_rope", x.data_ptr(), B, S, H, D, x.stride(0), x.stride(1), x.stride(2), table.data_ptr(),
                     ptr(pos), int(offset), -1.0 if inverse else 1.0, stream(x))
        return x
    x.copy_(rope_ref(x, table, positions, offset, inverse))
    return x


def rope_ref(x, table, positions=None, offset=0, inverse=False):
    B, S, H, D = x.shape
    half = D // 2
    if positions is None:
        positions = (torch.arange(S, device=x.device) + offset)[None, :].expand(B, S)
    cs = table.to(x.device)[positions.long()]  # [B, S, D]
    c, s = cs[..., :half][:, :, None, :], cs[..., half:][:, :, None, :]
    if inverse:
        s = -s
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


class _RopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, table, positions, offset):
        y = x.clone()
        apply_rope_(y, table, positions, offset)
        ctx.save_for_backward(table, positions) if positions is not None else ctx.save_for_backward(table)
        ctx.has_pos = positions is not None
        ctx.offset = offset
        return y

    @staticmethod
    def backward(ctx, dy):
        if ctx.has_pos:
            table, positions = ctx.saved_tensors
        else:
            (table,) = ctx.saved_tensors
            positions = None
        dx = dy.clone()
        apply_rope_(dx, table, positions, ctx.offset, inverse=True)
        return dx, None, None, None


def apply_rope(x, table, positions=None, offset=0):
    """Out-of-place, differentiable rotary embedding for x [B, S, H, D]."""
    if x.is_cuda:
        return _RopeFn.apply(x, table, positions, offset)
    return rope_ref(x, table, positions, offset)
