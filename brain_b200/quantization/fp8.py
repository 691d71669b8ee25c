"""FP8 E4M3 block-scaled quantisation and GEMM front-end (``csrc/fp8.cu``).

Activations: 1 x 128 blocks along K (scale = amax / 448 per row and block). Weights [N, K]:
128 x 128 blocks. ``fp8_gemm_blockscaled`` computes ``sum_kb (Aq . Bq^T) * sa * sb`` into bf16 on the
tcgen05 kernel; on CPU the same contract is evaluated by dequantising in float32 (the oracle).
"""
from __future__ import annotations

import torch

from .. import _native
from ..ops._common import ptr, stream

_native.register({
    "brain_fp8_gemm": ("brain_kernels", "plplppplpliiis"),
    "brain_fp8_quant_rows": ("brain_kernels", "plplpiis"),
    "brain_status_fp8": ("brain_kernels", "pi"),
})

E4M3_MAX = 448.0


def quantize_fp8_blockwise(x: torch.Tensor):
    """x [M, K] -> (q [M, K] float8_e4m3fn, scales [M, K/128] f32)."""
    M, K = x.shape
    if K % 128:
        raise ValueError("K must be a multiple of 128")
    if x.is_cuda and x.dtype == torch.bfloat16:
        xc = x if x.stride(1) == 1 else x.contiguous()
        q = torch.empty(M, K, device=x.device, dtype=torch.float8_e4m3fn)
        s = torch.empty(M, K // 128, device=x.device, dtype=torch.float32)
        _native.call("brain_fp8_quant_rows", xc.data_ptr(), xc.stride(0), q.data_ptr(), q.stride(0), s.data_ptr(),
                     M, K, stream(x))
        return q, s
    xb = x.float().view(M, K // 128, 128)
    s = (xb.abs().amax(-1) / E4M3_MAX)
    s = torch.where(s > 0, s, torch.ones_like(s))
    q = (xb / s[..., None]).to(torch.float8_e4m3fn).view(M, K)
    return q, s


def quantize_fp8_weight_blocks(w: torch.Tensor):
    """w [N, K] -> (q [N, K] e4m3, scales [ceil(N/128), K/128]) with 128 x 128 blocks."""
    N, K = w.shape
    if K % 128:
        raise ValueError("K must be a multiple of 128")
    Np = -(-N // 128) * 128
    wf = torch.zeros(Np, K, device=w.device, dtype=torch.float32)
    wf[:N] = w.float()
    blocks = wf.view(Np // 128, 128, K // 128, 128)
    s = blocks.abs().amax((1, 3)) / E4M3_MAX
    s = torch.where(s > 0, s, torch.ones_like(s))
    q = (blocks / s[:, None, :, None]).to(torch.float8_e4m3fn).view(Np, K)[:N].contiguous()
    return q, s.contiguous()


def dequantize_fp8_blockwise(q, s, block_rows: int = 1):
    """Inverse of either quantiser (block_rows 1 for activations, 128 for weights)."""
    M, K = q.shape
    sf = s.repeat_interleave(block_rows, 0)[:M] if block_rows > 1 else s
    return (q.float().view(M, K // 128, 128) * sf[..., None]).view(M, K)


def fp8_gemm_blockscaled(aq, sa, bq, sb, residual: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 C = dequant(aq, sa) @ dequant(bq, sb)^T (+ residual)."""
    M, K = aq.shape
    N = bq.shape[0]
    if aq.is_cuda:
        out = torch.empty(M, N, device=aq.device, dtype=torch.bfloat16)
        _native.call("brain_fp8_gemm", aq.data_ptr(), aq.stride(0), bq.data_ptr(), bq.stride(0), sa.data_ptr(),
                     sb.data_ptr(), out.data_ptr(), out.stride(0), ptr(residual),
                     residual.stride(0) if residual is not None else 0, M, N, K, stream(aq))
        return out
    a = dequantize_fp8_blockwise(aq, sa, 1)
    b = dequantize_fp8_blockwise(bq, sb, 128)
    c = a @ b.t()
    if residual is not None:
        c = c + residual.float()
    return c.to(torch.bfloat16)


def fp8_linear(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, residual=None) -> torch.Tensor:
    """y = x @ W^T with x quantised on the fly (1 x 128) and W pre-quantised (128 x 128)."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    aq, sa = quantize_fp8_blockwise(x2)
    r2 = residual.reshape(-1, wq.shape[0]) if residual is not None else None
    return fp8_gemm_blockscaled(aq, sa, wq, ws, r2).view(*shp[:-1], wq.shape[0])
