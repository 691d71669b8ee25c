"""GEMM front-end over the tcgen05 kernel (``csrc/gemm.cu``).

``gemm(a, b, trans_a, trans_b)`` computes ``op(a) @ op(b)`` with ``op(x) = x.T`` when the flag is
set, reading transposed operands in place (the kernel consumes MN-major shared-memory tiles), so
Linear forward, data-gradient and weight-gradient all run without transpose copies.
Epilogue options: ``alpha`` scaling, ``out`` accumulation (``beta * out``), ``bias`` [N] and a
``residual`` [M, N] added in the same pass.

On CPU tensors the same contract is evaluated with ``torch.matmul`` in float32 (the oracle path);
CUDA tensors always take the native kernel.
"""
from __future__ import annotations

import functools

import torch

from .. import _native
from ._common import same_device


def _row_major(x: torch.Tensor) -> torch.Tensor:
    if x.dim() != 2:
        raise ValueError("gemm operands must be 2-D")
    if x.stride(1) != 1 or x.stride(0) < x.size(1):
        x = x.contiguous()
    return x


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    trans_a: bool = False,
    trans_b: bool = False,
    *,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    alpha: float = 1.0,
    beta: float = 0.0,
    bias: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    force_simt: bool = False,
) -> torch.Tensor:
    """C = alpha * op(a) @ op(b) [+ beta * out] [+ bias] [+ residual].

    ``beta`` is only used when ``out`` is given (accumulation into an existing buffer).
    """
    a = _row_major(a)
    b = _row_major(b)
    M, K = (a.size(1), a.size(0)) if trans_a else (a.size(0), a.size(1))
    Kb, N = (b.size(1), b.size(0)) if trans_b else (b.size(0), b.size(1))
    if K != Kb:
        raise ValueError(f"gemm shape mismatch: op(a) is {M}x{K}, op(b) is {Kb}x{N}")
    accumulate = out is not None and beta != 0.0
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=out_dtype)
    if out.shape != (M, N):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {(M, N)}")
    if not a.is_cuda:
        return _gemm_cpu(a, b, trans_a, trans_b, out, alpha, beta if accumulate else 0.0, bias, residual)
    same_device(a, b, out, bias, residual)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("CUDA gemm takes bfloat16 operands")
    if out.dtype not in (torch.bfloat16, torch.float32) or out.stride(1) != 1:
        raise TypeError("gemm output must be row-major bfloat16 or float32")
    if bias is not None:
        bias = bias.contiguous()
        if bias.dtype != torch.bfloat16 or bias.numel() != N:
            raise TypeError("bias must be a bfloat16 vector of length N")
    if residual is not None:
        residual = _row_major(residual)
        if residual.dtype != torch.bfloat16 or residual.shape != (M, N):
            raise TypeError("residual must be bfloat16 [M, N]")
    splits = _splitk_plan(M, N, K) if (M >= 256 and N >= 256 and not force_simt) else 1
    if splits > 1:
        # few output tiles over a long K (weight gradients of narrow layers): K slices on separate SM
        # pairs into an f32 workspace, added in order by a second kernel
        ws = torch.empty(splits * ((M + 255) // 256) * 256 * N, device=a.device, dtype=torch.float32)
        _native.call(
            "brain_gemm_bf16_ws",
            a.data_ptr(), a.stride(0), int(trans_a),
            b.data_ptr(), b.stride(0), int(not trans_b),
            out.data_ptr(), out.stride(0), int(out.dtype == torch.float32),
            M, N, K, float(alpha), int(accumulate), float(beta),
            bias.data_ptr() if bias is not None else None,
            residual.data_ptr() if residual is not None else None,
            residual.stride(0) if residual is not None else 0,
            ws.data_ptr(), ws.numel(),
            _native.stream_ptr(a.device),
        )
        return out
    _native.call(
        "brain_gemm_bf16",
        a.data_ptr(), a.stride(0), int(trans_a),
        b.data_ptr(), b.stride(0), int(not trans_b),
        out.data_ptr(), out.stride(0), int(out.dtype == torch.float32),
        M, N, K, float(alpha), int(accumulate), float(beta),
        bias.data_ptr() if bias is not None else None,
        residual.data_ptr() if residual is not None else None,
        residual.stride(0) if residual is not None else 0,
        int(force_simt),
        _native.stream_ptr(a.device),
    )
    return out


_NOT_SUPPORTED = 801  # cudaErrorNotSupported
_SPLIT_ON = {"on": True}


@functools.lru_cache(maxsize=4096)
def _plan(M: int, N: int, K: int) -> int:
    return int(_native.fn("brain_gemm_splitk_plan")(M, N, K, None))


def _splitk_plan(M: int, N: int, K: int) -> int:
    """Number of K slices the CTA-pair kernel uses for this shape (1: no split). Only shapes with fewer
    256 x 256 output tiles than SM pairs and at least 16 k-blocks are split."""
    if not _SPLIT_ON["on"] or K < 1024:
        return 1
    return _plan(M, N, K)


def set_splitk(on: bool) -> bool:
    """Enable or disable split-K for under-filled GEMMs (tests compare both); returns the previous state."""
    old = _SPLIT_ON["on"]
    _SPLIT_ON["on"] = bool(on)
    return old


def gemm_rope(x: torch.Tensor, w: torch.Tensor, table: torch.Tensor, rope_cols: int, head_dim: int, seq_len: int,
              offset: int = 0) -> torch.Tensor | None:
    """y = x @ w.T (bf16) with NeoX RoPE applied in the GEMM epilogue to the first ``rope_cols`` output
    columns (the q and k heads of a fused QKV projection, heads of ``head_dim``); row r of x is token
    (r % seq_len) + offset; ``table`` is the f32 [positions, head_dim] cos | sin table of ``ops.rope``.
    Returns None where the fused epilogue does not apply (small or unaligned shapes): the caller then
    rotates separately."""
    if not x.is_cuda or x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or table.dtype != torch.float32:
        return None
    x = _row_major(x)
    w = _row_major(w)
    if x.stride(1) != 1 or w.stride(1) != 1 or not table.is_contiguous():
        return None
    same_device(x, w, table)
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    rc = _native.fn("brain_gemm_bf16_rope")(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
                                            out.stride(0), M, N, K, table.data_ptr(), int(rope_cols), int(head_dim),
                                            int(seq_len), int(offset), _native.stream_ptr(x.device))
    if rc == _NOT_SUPPORTED:
        return None
    if rc != 0:
        raise _native.NativeError(f"brain_gemm_bf16_rope failed with status {rc}")
    return out


def set_pair_mode(mode: int) -> int:
    """1: use the CTA-pair (cta_group::2, 256x256 tile) kernel for M, N >= 256; 0: single-CTA
    kernel only. Returns the previous mode."""
    return int(_native.fn("brain_gemm_set_pair_mode")(int(mode)))


def _gemm_cpu(a, b, ta, tb, out, alpha, beta, bias, residual):
    A = a.float().t() if ta else a.float()
    B = b.float().t() if tb else b.float()
    r = alpha * (A @ B)
    if beta:
        r = r + beta * out.float()
    if bias is not None:
        r = r + bias.float()
    if residual is not None:
        r = r + residual.float()
    out.copy_(r.to(out.dtype))
    return out


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
           residual: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w.T (+ bias) (+ residual) for x [..., K] and a [N, K] weight."""
    shp = x.shape
    y = gemm(x.reshape(-1, shp[-1]), w, trans_b=True, bias=bias,
             residual=None if residual is None else residual.reshape(-1, w.size(0)),
             out_dtype=x.dtype if not x.is_cuda else torch.bfloat16)
    return y.reshape(*shp[:-1], w.size(0))
