"""Helpers shared by the op modules: signatures, streams, parameter-gradient accumulation."""
from __future__ import annotations

import ctypes

import torch

from .. import _native

# Signatures of the kernel entry points (see csrc/*.cu). Codes: p pointer, i int32, l int64,
# f float32, s cudaStream_t.
_native.register({
    "brain_norm_fwd": ("brain_kernels", "iplplppplplppiifs"),
    "brain_norm_bwd_partials": ("brain_kernels", "i"),
    "brain_colsum_partials": ("brain_kernels", "i"),
    "brain_colsum_bf16": ("brain_kernels", "pliipiips"),
    "brain_gemm_bf16_gelu_dual": ("brain_kernels", "plplplpliiips"),
    "brain_gemm_bf16_gelu_grad": ("brain_kernels", "plpliplpliiis"),
    "brain_norm_bwd": ("brain_kernels", "iplplpppplplppiipiis"),
    "brain_swiglu_fwd": ("brain_kernels", "plpllis"),
    "brain_swiglu_bwd": ("brain_kernels", "plplpllis"),
    "brain_gelu_fwd": ("brain_kernels", "ppls"),
    "brain_gelu_bwd": ("brain_kernels", "pppls"),
    "brain_rope": ("brain_kernels", "piiiilllppifs"),
    "brain_embedding_fwd": ("brain_kernels", "pppiplils"),
    "brain_embedding_bwd": ("brain_kernels", "ppppilils"),
    "brain_pos_grad": ("brain_kernels", "ppilii" + "s"),
    "brain_ce_fwd": ("brain_kernels", "plppplilfs"),
    "brain_ce_bwd": ("brain_kernels", "plppppfpllilfs"),
    "brain_adamw": ("brain_kernels", "pppppiplffffffffipps"),
    "brain_grad_stats": ("brain_kernels", "pilfpips"),
    "brain_step_guard": ("brain_kernels", "pfpps"),
    "brain_sgd": ("brain_kernels", "pppiplffffiifps"),
    "brain_sumsq": ("brain_kernels", "pilfpipps"),
    "brain_scale": ("brain_kernels", "pilpfs"),
    "brain_clip_coef": ("brain_kernels", "pfps"),
    "brain_cast_bf16": ("brain_kernels", "ppls"),
    "brain_attn_fwd": ("brain_kernels", "pppppppiiiiiifis"),
    "brain_attn_bwd": ("brain_kernels", "pppppppppppppppp" + "iiiiiifis"),
    "brain_attn_fwd_tc": ("brain_kernels", "pppppppiiiiiifis"),
    "brain_status_attention_tc": ("brain_kernels", "pi"),
    "brain_attn_bwd_tc": ("brain_kernels", "pppppppppppppppp" + "iiiiiifis"),
    "brain_attn_fwd_tc_masked": ("brain_kernels", "pppppppiiiiiifipps"),
    "brain_attn_bwd_tc_masked": ("brain_kernels", "pppppppppppppppp" + "iiiiiifipps"),
    "brain_status_attention_bwd_tc": ("brain_kernels", "pi"),
    "brain_status_norms": ("brain_kernels", "pi"),
    "brain_status_elementwise": ("brain_kernels", "pi"),
    "brain_status_ce": ("brain_kernels", "pi"),
    "brain_status_optim": ("brain_kernels", "pi"),
    "brain_status_attention": ("brain_kernels", "pi"),
})

STATUS_TAGS = ["gemm", "norms", "elementwise", "ce", "optim", "attention", "attention_tc", "attention_bwd_tc",
               "attention_decode", "decode_tp"]


def same_device(ref: torch.Tensor, *others) -> None:
    """Raise unless every tensor in ``others`` (None skipped) lives on ``ref``'s device: a kernel given a
    pointer into another device's (or the host's) memory would fault."""
    for t in others:
        if t is not None and t.device != ref.device:
            raise ValueError(f"tensor on {t.device} passed to a kernel running on {ref.device}")


def stream(t: torch.Tensor) -> int:
    return _native.stream_ptr(t.device)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def i64_array(vals) -> ctypes.Array:
    arr = (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])
    return arr


def check_status() -> list[tuple[str, int, int]]:
    """Read and clear every kernel status word; returns the non-zero entries (tag, code, where)."""
    bad = []
    for tag in STATUS_TAGS:
        code, where = _native.status(tag, clear=True)
        if code:
            bad.append((tag, code, where))
    return bad


def has_main_grad(p: torch.Tensor) -> bool:
    return getattr(p, "main_grad", None) is not None


def main_grad_beta(p: torch.Tensor) -> float:
    """Weight of the existing contents of ``p.main_grad`` for the next gradient written into it: 0.0
    for the first write since the flat buffer's ``zero_grad`` (which marks parameters instead of
    clearing memory, so the first producer overwrites), 1.0 afterwards (accumulate)."""
    if getattr(p, "_main_grad_fresh", False):
        p._main_grad_fresh = False
        return 0.0
    return 1.0


def rows2d(x: torch.Tensor) -> torch.Tensor:
    """View x as [rows, last] with unit last-dim stride (copying only if needed)."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2
