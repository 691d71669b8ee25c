"""Flat parameter / gradient storage shared by the optimizer and the data-parallel engine.

All trainable parameters of a model are re-pointed into one contiguous bf16 buffer (``param.data``
becomes a view), and every parameter gets a ``main_grad`` view into one flat gradient buffer. The
GEMM weight-gradient epilogues, the norm kernels and the embedding backward accumulate straight
into ``main_grad`` (see ``ops.linear``), so backward produces the gradient bucket directly in the
layout the collectives and the fused optimizer consume: no per-parameter ``.grad`` tensors, no
copies into communication buffers.

The buffer is padded to a multiple of ``world_size * align`` so that every rank owns an equal,
16-byte-aligned shard (ZeRO-1 style optimizer sharding).
"""
from __future__ import annotations

import torch


class FlatParams:
    def __init__(self, params: list[torch.nn.Parameter], world_size: int = 1, rank: int = 0,
                 grad_dtype: torch.dtype = torch.float32, align: int = 64, alloc=None):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        dev = self.params[0].device
        dtype = self.params[0].dtype
        self.world_size, self.rank = world_size, rank
        self.offsets = []
        off = 0
        for p in self.params:
            self.offsets.append(off)
            off += -(-p.numel() // align) * align  # keep every parameter 16-byte aligned
        self.numel = off
        unit = world_size * align
        self.padded = -(-off // unit) * unit
        self.shard_size = self.padded // world_size
        if alloc is None:  # plain device memory; the NVLink backend passes a symmetric allocator
            def alloc(n, dt):
                return torch.zeros(n, device=dev, dtype=dt)
        self.param_buf = alloc(self.padded, dtype)
        self.grad_buf = alloc(self.padded, grad_dtype)
        with torch.no_grad():
            for p, o in zip(self.params, self.offsets):
                n = p.numel()
                self.param_buf[o:o + n].copy_(p.data.reshape(-1))
                p.data = self.param_buf[o:o + n].view(p.shape)
                p.main_grad = self.grad_buf[o:o + n].view(p.shape)
                p.grad = None

    # shard of this rank ---------------------------------------------------------------
    def shard(self, buf: torch.Tensor, rank: int | None = None) -> torch.Tensor:
        r = self.rank if rank is None else rank
        return buf[r * self.shard_size:(r + 1) * self.shard_size]

    def zero_grad(self) -> None:
        """Restart every gradient from zero without clearing memory: each parameter is marked fresh,
        its first gradient producer overwrites its ``main_grad`` (``ops._common.main_grad_beta``), and
        ``finalize_grads`` zeroes the parameters no producer wrote."""
        for p in self.params:
            p.grad = None
            p._main_grad_fresh = True

    def params_in(self, lo: int, hi: int) -> list:
        """Parameters overlapping flat range [lo, hi)."""
        return [p for p, o in zip(self.params, self.offsets) if o < hi and o + p.numel() > lo]

    @torch.no_grad()
    def finalize_grads(self, params=None) -> None:
        """Zero the gradients still marked fresh (no producer wrote them since ``zero_grad``) among
        ``params`` (default: all)."""
        for p in (self.params if params is None else params):
            if getattr(p, "_main_grad_fresh", False):
                p.main_grad.zero_()
                p._main_grad_fresh = False

    @torch.no_grad()
    def absorb_grads(self) -> None:
        """Fold gradients that reached ``param.grad`` (ops without a main_grad path, CPU
        reference ops, user code) into the flat buffer, then zero what nothing wrote."""
        for p in self.params:
            if p.grad is not None:
                if getattr(p, "_main_grad_fresh", False):
                    p.main_grad.copy_(p.grad.to(p.main_grad.dtype))
                    p._main_grad_fresh = False
                else:
                    p.main_grad.add_(p.grad.to(p.main_grad.dtype))
                p.grad = None
        self.finalize_grads()

    def param_ranges(self, lo: int, hi: int):
        """(param, start, end) pieces of parameters overlapping flat range [lo, hi)."""
        for p, o in zip(self.params, self.offsets):
            s, e = max(lo, o), min(hi, o + p.numel())
            if s < e:
                yield p, s - o, e - o

    def no_decay_mask(self, shard_only: bool = True) -> torch.Tensor | None:
        """1.0 where weight decay applies (matrices), 0.0 for vectors (norms, biases)."""
        lo, hi = (self.rank * self.shard_size, (self.rank + 1) * self.shard_size) if shard_only else (0, self.padded)
        mask = torch.zeros(hi - lo, device=self.param_buf.device, dtype=torch.float32)
        for p, o in zip(self.params, self.offsets):
            if p.dim() >= 2:
                s, e = max(lo, o), min(hi, o + p.numel())
                if s < e:
                    mask[s - lo:e - lo] = 1.0
        return mask
