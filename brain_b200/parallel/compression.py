"""Gradient compression (reference enum ``CompressionType::{None, TopK, Quantize8Bit}`` with a stub
``topk_compress``, crates/brain-distributed/src/grad_compression.rs:9-18).

* top-k sparsification with error feedback (the residual of what was not sent is added back next step);
* 8-bit quantisation with a per-chunk absmax scale.
``compressed_all_reduce`` all-gathers the compressed payloads and decompresses / sums locally.
"""
from __future__ import annotations

import enum

import torch
import torch.distributed as dist


class CompressionType(enum.Enum):
    NONE = 0
    TOPK = 1
    QUANTIZE_8BIT = 2


def topk_compress(g: torch.Tensor, ratio: float):
    flat = g.reshape(-1)
    k = max(1, int(flat.numel() * ratio))
    vals, idx = flat.abs().topk(k)
    return flat[idx], idx


def topk_decompress(vals, idx, numel, dtype=torch.float32, device=None):
    out = torch.zeros(numel, dtype=dtype, device=device or vals.device)
    out.index_add_(0, idx, vals.to(dtype))
    return out


def quantize_int8(g: torch.Tensor, chunk: int = 2048):
    flat = g.reshape(-1).float()
    pad = (-flat.numel()) % chunk
    x = torch.nn.functional.pad(flat, (0, pad)).view(-1, chunk)
    scale = x.abs().amax(1).clamp_min(1e-12) / 127.0
    q = torch.round(x / scale[:, None]).clamp(-127, 127).to(torch.int8)
    return q, scale, flat.numel()


def dequantize_int8(q, scale, numel):
    return (q.float() * scale[:, None]).reshape(-1)[:numel]


class ErrorFeedback:
    """Keeps the per-tensor residual of lossy compression and adds it back before compressing."""

    def __init__(self):
        self.residual: dict = {}

    def compress_topk(self, key, g, ratio):
        r = self.residual.get(key)
        x = g.float() + (r if r is not None else 0)
        vals, idx = topk_compress(x, ratio)
        sent = topk_decompress(vals, idx, x.numel(), device=x.device).view_as(x)
        self.residual[key] = x - sent
        return vals, idx


def compressed_all_reduce(g: torch.Tensor, kind: CompressionType, ratio: float = 0.01, group=None) -> torch.Tensor:
    """Mean over ranks of g using the chosen compression; returns a new tensor."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1 or kind == CompressionType.NONE:
        out = g.clone()
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(out, group=group)
            out /= dist.get_world_size(group)
        return out
    w = dist.get_world_size(group)
    if kind == CompressionType.TOPK:
        vals, idx = topk_compress(g, ratio)
        vs = [torch.empty_like(vals) for _ in range(w)]
        ix = [torch.empty_like(idx) for _ in range(w)]
        dist.all_gather(vs, vals, group=group)
        dist.all_gather(ix, idx, group=group)
        out = torch.zeros(g.numel(), dtype=torch.float32, device=g.device)
        for v, i in zip(vs, ix):
            out.index_add_(0, i, v.float())
        return (out / w).view_as(g).to(g.dtype)
    q, s, n = quantize_int8(g)
    qs = [torch.empty_like(q) for _ in range(w)]
    ss = [torch.empty_like(s) for _ in range(w)]
    dist.all_gather(qs, q, group=group)
    dist.all_gather(ss, s, group=group)
    out = sum(dequantize_int8(a, b, n) for a, b in zip(qs, ss))
    return (out / w).view_as(g).to(g.dtype)
