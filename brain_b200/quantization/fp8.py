"""FP8 E4M3 quantisation and GEMM front-ends (``csrc/fp8.cu``, ``csrc/gemm.cu``).

Block-scaled: activations in 1 x 128 blocks along K (scale = amax / 448 per row and block), weights
[N, K] in 128 x 128 blocks; ``fp8_gemm_blockscaled`` computes ``sum_kb (Aq . Bq^T) * sa * sb`` into
bf16, promoting each 128-wide K block on the CUDA cores.

Row-wise: one scale per activation row (token) and one per weight row (output channel);
``fp8_gemm_rowwise`` accumulates the whole K reduction on the tensor core (tcgen05 kind::f8f6f4,
256 x 256 CTA-pair tiles, the bf16 GEMM's pipeline) and applies ``sa[m] * sb[n]`` once in the epilogue,
so it runs at the fp8 tensor rate. Coarser scales than the block-scaled path (an outlier costs its
whole row or channel precision), the usual trade of a row-wise fp8 training / serving recipe.

On CPU both contracts are evaluated by dequantising in float32 (the oracle).
"""
from __future__ import annotations

import torch

from .. import _native
from ..ops._common import ptr, stream

_native.register({
    "brain_fp8_gemm": ("brain_kernels", "plplppplpliiis"),
    "brain_fp8_quant_rows": ("brain_kernels", "plplpiis"),
    "brain_status_fp8": ("brain_kernels", "pi"),
    "brain_fp8_gemm_rowwise": ("brain_kernels", "plplppplpliiis"),
    "brain_fp8_gemm_rowwise_pair": ("brain_kernels", "plplppplpliiis"),
    "brain_fp8_quant_rowwise": ("brain_kernels", "plplpiis"),
})
_NOT_SUPPORTED = 801  # cudaErrorNotSupported

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


# ------------------------------------------------------------------ row-wise scaling
def _aligned_rows(t: torch.Tensor) -> torch.Tensor:
    """t itself when its rows are unit-stride, 16-byte aligned and a multiple of 8 elements apart, else a
    copy into such a buffer (a view of its first N columns)."""
    if t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0:
        return t
    M, N = t.shape
    buf = torch.empty(M, -(-N // 8) * 8, device=t.device, dtype=t.dtype)[:, :N]
    buf.copy_(t)
    return buf


def quantize_fp8_rowwise(x: torch.Tensor):
    """x [M, K] -> (q [M, K] float8_e4m3fn, scales [M] f32), scale = amax(|row|) / 448."""
    M, K = x.shape
    if x.is_cuda and x.dtype == torch.bfloat16 and K % 8 == 0:
        xc = x if (x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0) else x.contiguous()
        q = torch.empty(M, K, device=x.device, dtype=torch.float8_e4m3fn)
        s = torch.empty(M, device=x.device, dtype=torch.float32)
        _native.call("brain_fp8_quant_rowwise", xc.data_ptr(), xc.stride(0), q.data_ptr(), q.stride(0), s.data_ptr(),
                     M, K, stream(x))
        return q, s
    xf = x.float()
    s = xf.abs().amax(-1) / E4M3_MAX
    s = torch.where(s > 0, s, torch.ones_like(s))
    return (xf / s[:, None]).to(torch.float8_e4m3fn), s


def fp8_gemm_rowwise(aq, sa, bq, sb, residual: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 C = (aq . bq^T) * sa[:, None] * sb[None, :] (+ residual): the CTA-pair tcgen05 kernel for
    M, N >= 256, the single-CTA 128 x 256 kernel otherwise."""
    M, K = aq.shape
    N = bq.shape[0]
    if aq.is_cuda:
        if K % 16 or aq.stride(1) != 1 or bq.stride(1) != 1:
            raise ValueError("fp8_gemm_rowwise needs K % 16 == 0 and row-major operands")
        sa = sa.float().contiguous()
        sb = sb.float().contiguous()
        ld = -(-N // 8) * 8  # 16-byte output rows for the vector / TMA stores
        out = torch.empty(M, ld, device=aq.device, dtype=torch.bfloat16)[:, :N]
        if residual is not None:
            residual = _aligned_rows(residual.to(torch.bfloat16))
        args = (aq.data_ptr(), aq.stride(0), bq.data_ptr(), bq.stride(0), sa.data_ptr(), sb.data_ptr(),
                out.data_ptr(), out.stride(0), ptr(residual), residual.stride(0) if residual is not None else 0,
                M, N, K, stream(aq))
        rc = _native.fn("brain_fp8_gemm_rowwise_pair")(*args)
        if rc == _NOT_SUPPORTED:
            rc = _native.fn("brain_fp8_gemm_rowwise")(*args)
        if rc != 0:
            raise _native.NativeError(f"fp8 row-wise GEMM failed with status {rc}")
        return out
    c = (aq.float() * sa.float()[:, None]) @ (bq.float() * sb.float()[:, None]).t()
    if residual is not None:
        c = c + residual.float()
    return c.to(torch.bfloat16)


def fp8_linear_rowwise(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, residual=None) -> torch.Tensor:
    """y = x @ W^T with x quantised per token on the fly and W quantised per output channel
    (``quantize_fp8_rowwise(w)``)."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    aq, sa = quantize_fp8_rowwise(x2)
    r2 = residual.reshape(-1, wq.shape[0]) if residual is not None else None
    return fp8_gemm_rowwise(aq, sa, wq, ws, r2).view(*shp[:-1], wq.shape[0])


class Fp8Linear(torch.nn.Module):
    """Inference Linear with e4m3 weights: ``scaling="rowwise"`` (one scale per output channel; tokens
    quantised per row on the fly; the CTA-pair fp8 kernel) or ``"block"`` (128 x 128 weight blocks,
    1 x 128 activation blocks). Built from a float Linear with ``from_linear``; the bias is added in
    bf16 after the GEMM."""

    def __init__(self, wq: torch.Tensor, ws: torch.Tensor, bias: torch.Tensor | None = None, scaling: str = "rowwise"):
        super().__init__()
        if scaling not in ("rowwise", "block"):
            raise ValueError(f"unknown fp8 scaling {scaling!r}")
        self.scaling = scaling
        self.register_buffer("wq", wq)
        self.register_buffer("ws", ws)
        self.register_buffer("bias", bias)
        self.out_features, self.in_features = wq.shape

    @classmethod
    def from_linear(cls, lin: torch.nn.Module, scaling: str = "rowwise") -> "Fp8Linear":
        w = lin.weight.detach()
        wq, ws = quantize_fp8_rowwise(w.to(torch.bfloat16) if w.is_cuda else w) if scaling == "rowwise" \
            else quantize_fp8_weight_blocks(w)
        b = lin.bias.detach().to(torch.bfloat16) if getattr(lin, "bias", None) is not None else None
        return cls(wq, ws, b, scaling)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        f = fp8_linear_rowwise if self.scaling == "rowwise" else fp8_linear
        y = f(x.to(torch.bfloat16) if x.is_cuda else x, self.wq, self.ws, residual)
        return y + self.bias if self.bias is not None else y
