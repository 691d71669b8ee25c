"""Float64 CPU oracle kernels in C++ (``csrc/oracle.cpp``, in ``libbrain_runtime``): GEMM, RMSNorm,
LayerNorm, softmax, cross-entropy, NeoX RoPE and GQA attention with bottom-right causal masking,
following the reference's f64 definitions. Tests compare the GPU kernels and the PyTorch float64
restatements against them; inputs are converted to contiguous float64 CPU tensors."""
from __future__ import annotations

import torch

from . import _native

_native.register({
    "brain_oracle_gemm": ("brain_runtime", "ppplll"),
    "brain_oracle_rms_norm": ("brain_runtime", "ppplld"),
    "brain_oracle_layer_norm": ("brain_runtime", "pppplld"),
    "brain_oracle_softmax": ("brain_runtime", "ppll"),
    "brain_oracle_cross_entropy": ("brain_runtime", "ppplll"),
    "brain_oracle_rope": ("brain_runtime", "pllldl"),
    "brain_oracle_attention": ("brain_runtime", "ppppllllli"),
})


def _d(t) -> torch.Tensor:
    return torch.as_tensor(t).detach().to("cpu", torch.float64).contiguous()


def gemm_nt(a, b) -> torch.Tensor:
    """a [M, K] @ b[N, K]^T."""
    a, b = _d(a), _d(b)
    c = torch.empty(a.shape[0], b.shape[0], dtype=torch.float64)
    _native.call("brain_oracle_gemm", a.data_ptr(), b.data_ptr(), c.data_ptr(), a.shape[0], b.shape[0], a.shape[1])
    return c


def rms_norm(x, w, eps: float = 1e-6) -> torch.Tensor:
    x, w = _d(x), _d(w)
    y = torch.empty_like(x)
    D = x.shape[-1]
    _native.call("brain_oracle_rms_norm", x.data_ptr(), w.data_ptr(), y.data_ptr(), x.numel() // D, D, float(eps))
    return y


def layer_norm(x, w, b=None, eps: float = 1e-5) -> torch.Tensor:
    x, w = _d(x), _d(w)
    bb = _d(b) if b is not None else None
    y = torch.empty_like(x)
    D = x.shape[-1]
    _native.call("brain_oracle_layer_norm", x.data_ptr(), w.data_ptr(), bb.data_ptr() if bb is not None else None,
                 y.data_ptr(), x.numel() // D, D, float(eps))
    return y


def softmax(x) -> torch.Tensor:
    x = _d(x)
    y = torch.empty_like(x)
    N = x.shape[-1]
    _native.call("brain_oracle_softmax", x.data_ptr(), y.data_ptr(), x.numel() // N, N)
    return y


def cross_entropy(logits, labels, ignore_index: int = -100) -> torch.Tensor:
    """Mean over the rows whose label is not ``ignore_index``."""
    lg = _d(logits)
    lab = torch.as_tensor(labels).to("cpu", torch.int64).contiguous()
    loss = torch.empty(lg.shape[0], dtype=torch.float64)
    _native.call("brain_oracle_cross_entropy", lg.data_ptr(), lab.data_ptr(), loss.data_ptr(), lg.shape[0],
                 lg.shape[1], int(ignore_index))
    n = int((lab != ignore_index).sum())
    return loss.sum() / max(1, n)


def rope(x, theta: float = 10000.0, offset: int = 0) -> torch.Tensor:
    """x [S, H, D] (or [B, S, H, D]), NeoX rotation; returns a rotated copy."""
    y = _d(x).clone()
    if y.dim() == 4:
        return torch.stack([rope(b, theta, offset) for b in y])
    S, H, D = y.shape
    _native.call("brain_oracle_rope", y.data_ptr(), S, H, D, float(theta), int(offset))
    return y


def attention(q, k, v, causal: bool = True) -> torch.Tensor:
    """q [B, Sq, Hq, D], k / v [B, Sk, Hkv, D] -> [B, Sq, Hq, D]."""
    q, k, v = _d(q), _d(k), _d(v)
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    o = torch.empty_like(q)
    for b in range(B):
        qb, kb, vb, ob = q[b].contiguous(), k[b].contiguous(), v[b].contiguous(), o[b]
        _native.call("brain_oracle_attention", qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), ob.data_ptr(), Sq, Sk,
                     Hq, Hkv, D, int(causal))
    return o
