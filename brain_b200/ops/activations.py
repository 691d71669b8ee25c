"""SwiGLU and tanh-GELU ops (``csrc/elementwise.cu``).

SwiGLU = silu(gate) * up (crates/brain-core/src/tensor/ops_fused.rs:127-142) over a fused
``[..., 2F]`` gate/up projection (gate first). GELU is the tanh approximation used everywhere in
the reference (crates/brain-core/src/tensor/math.rs:284-287).
"""
from __future__ import annotations

import math

import torch

from .. import _native
from ._common import rows2d, stream


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        g2 = rows2d(gu)
        M, F2 = g2.shape
        F = F2 // 2
        out = torch.empty(M, F, device=gu.device, dtype=gu.dtype)
        _native.call("brain_swiglu_fwd", g2.data_ptr(), g2.stride(0), out.data_ptr(), out.stride(0), M, F, stream(gu))
        ctx.save_for_backward(g2)
        ctx.shape = gu.shape
        return out.view(*gu.shape[:-1], F)

    @staticmethod
    def backward(ctx, dy):
        (g2,) = ctx.saved_tensors
        M, F2 = g2.shape
        dy2 = rows2d(dy)
        dgu = torch.empty_like(g2)
        _native.call("brain_swiglu_bwd", dy2.data_ptr(), dy2.stride(0), g2.data_ptr(), g2.stride(0), dgu.data_ptr(),
                     dgu.stride(0), M, F2 // 2, stream(dy))
        return dgu.view(ctx.shape)


def swiglu_ref(gu: torch.Tensor) -> torch.Tensor:
    g, u = gu.float().chunk(2, dim=-1)
    return (torch.nn.functional.silu(g) * u).to(gu.dtype)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """silu(gu[..., :F]) * gu[..., F:]."""
    if gu.is_cuda:
        return _SwiGLUFn.apply(gu)
    return swiglu_ref(gu)


def swiglu_fwd_only(gu2: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """No-autograd SwiGLU on a 2-D [M, 2F] CUDA tensor (used by fused ops that recompute)."""
    M, F2 = gu2.shape
    if out is None:
        out = torch.empty(M, F2 // 2, device=gu2.device, dtype=gu2.dtype)
    _native.call("brain_swiglu_fwd", gu2.data_ptr(), gu2.stride(0), out.data_ptr(), out.stride(0), M, F2 // 2,
                 stream(gu2))
    return out


def swiglu_bwd_only(dy2, gu2, dgu=None):
    M, F2 = gu2.shape
    if dgu is None:
        dgu = torch.empty_like(gu2)
    _native.call("brain_swiglu_bwd", dy2.data_ptr(), dy2.stride(0), gu2.data_ptr(), gu2.stride(0), dgu.data_ptr(),
                 dgu.stride(0), M, F2 // 2, stream(gu2))
    return dgu


class _GeluFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        xc = x.contiguous()
        y = torch.empty_like(xc)
        _native.call("brain_gelu_fwd", xc.data_ptr(), y.data_ptr(), xc.numel(), stream(x))
        ctx.save_for_backward(xc)
        return y

    @staticmethod
    def backward(ctx, dy):
        (xc,) = ctx.saved_tensors
        dyc = dy.contiguous()
        dx = torch.empty_like(xc)
        _native.call("brain_gelu_bwd", dyc.data_ptr(), xc.data_ptr(), dx.data_ptr(), xc.numel(), stream(dy))
        return dx


def gelu_ref(x: torch.Tensor) -> torch.Tensor:
    xf = x.float()
    y = 0.5 * xf * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (xf + 0.044715 * xf.pow(3))))
    return y.to(x.dtype)


def gelu(x: torch.Tensor) -> torch.Tensor:
    """tanh-approximate GELU."""
    if x.is_cuda and x.dtype == torch.bfloat16:
        return _GeluFn.apply(x)
    return gelu_ref(x)
