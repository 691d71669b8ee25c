"""``LinearParams``: the reference transformer's projection container, in its own layout and init.

The reference keeps a projection as ``weight [in_features, out_features]`` plus an optional zero bias
and computes ``Y = X W + b`` (crates/brain-transformer/src/core.rs:110-191). Its weights are initialised
without a random generator, from the position of each element:
    s   = (seed + (i * 10007 + j * 37 + 1)) as f64            (u64 wrapping add)
    w_ij = fract(sin(s) * 43758.5453) * 2 * std - std,        std = sqrt(2 / (in + out))
with ``fract`` keeping the sign (x - trunc(x)). This module reproduces that init and layout, so that a
run seeded like the reference starts from the same weights, and it converts between the reference
layout and this framework's ``[out_features, in_features]`` Linear weights (``to_linear_weight`` /
``from_linear_weight``; ``load_into`` copies into a ``torch.nn.Linear`` or a raw weight parameter).

On a CUDA device the forward is the tcgen05 GEMM reading the ``[in, out]`` weight in place as an
MN-major operand (no transpose); on the CPU it is a float64/float32 matmul.

``exact=True`` evaluates ``sin`` per element with the C library (``math.sin``), as the reference
does on Linux, so the values are bit-identical to the reference's; the default vectorised float64
path differs from them by at most a few units in the 11th decimal place (``sin`` rounding amplified
by the 43758.5453 factor before ``fract``).
"""
from __future__ import annotations

import math

import torch

_U64 = 1 << 64


def reference_init(in_features: int, out_features: int, seed: int, exact: bool = False) -> torch.Tensor:
    """float64 ``[in_features, out_features]`` weights of ``LinearParams::new`` with ``seed``."""
    std = math.sqrt(2.0 / (in_features + out_features))
    if exact:
        vals = []
        for i in range(in_features):
            for j in range(out_features):
                s = float((seed + i * 10007 + j * 37 + 1) % _U64)
                x = math.sin(s) * 43758.5453
                vals.append((x - math.trunc(x)) * 2.0 * std - std)
        return torch.tensor(vals, dtype=torch.float64).view(in_features, out_features)
    i = torch.arange(in_features, dtype=torch.int64)[:, None]
    j = torch.arange(out_features, dtype=torch.int64)[None, :]
    # seed + index stays far below 2^63 for any layer size; the u64 wrap only matters for huge seeds
    idx = i * 10007 + j * 37 + 1
    if seed >= (1 << 62):
        s = torch.tensor([float((seed + int(v)) % _U64) for v in idx.flatten()], dtype=torch.float64)
        s = s.view(in_features, out_features)
    else:
        s = (idx + int(seed)).to(torch.float64)
    x = torch.sin(s) * 43758.5453
    return (x - torch.trunc(x)) * 2.0 * std - std


class LinearParams(torch.nn.Module):
    """Projection with the reference's ``[in, out]`` weight and position-hash initialisation."""

    def __init__(self, in_features: int, out_features: int, has_bias: bool = False, seed: int = 0, device=None,
                 dtype=torch.float32, exact: bool = False):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        w = reference_init(in_features, out_features, seed, exact)
        self.weight = torch.nn.Parameter(w.to(device=device, dtype=dtype))
        self.bias = torch.nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype)) if has_bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features:
            raise ValueError(f"LinearParams: expected last dimension {self.in_features}, found {x.shape[-1]}")
        if x.is_cuda and x.dtype == torch.bfloat16 and self.weight.dtype == torch.bfloat16:
            from ..ops.gemm import gemm
            x2 = x.reshape(-1, self.in_features)
            y = gemm(x2.contiguous(), self.weight, bias=self.bias)
            return y.view(*x.shape[:-1], self.out_features)
        y = x.to(self.weight.dtype) @ self.weight
        return y + self.bias if self.bias is not None else y

    # ---- layout conversion -----------------------------------------------------------------
    def to_linear_weight(self) -> torch.Tensor:
        """The weight as ``[out_features, in_features]`` (this framework's Linear layout)."""
        return self.weight.detach().t().contiguous()

    @staticmethod
    def from_linear_weight(w: torch.Tensor, bias: torch.Tensor | None = None) -> "LinearParams":
        out_f, in_f = w.shape
        lp = LinearParams(in_f, out_f, bias is not None, device=w.device, dtype=w.dtype)
        with torch.no_grad():
            lp.weight.copy_(w.t())
            if bias is not None:
                lp.bias.copy_(bias)
        return lp

    @torch.no_grad()
    def load_into(self, target) -> None:
        """Copy into a ``torch.nn.Linear`` (weight and bias) or an ``[out, in]`` weight parameter."""
        w = self.to_linear_weight()
        if isinstance(target, torch.nn.Linear):
            target.weight.copy_(w.to(target.weight.dtype))
            if target.bias is not None:
                target.bias.copy_(self.bias if self.bias is not None else torch.zeros_like(target.bias))
            return
        if tuple(target.shape) != tuple(w.shape):
            raise ValueError(f"target shape {tuple(target.shape)} != [out, in] {tuple(w.shape)}")
        target.copy_(w.to(target.dtype))


def load_reference_projection(target, weight_in_out: torch.Tensor, bias: torch.Tensor | None = None) -> None:
    """Load a reference-layout ``[in, out]`` weight (e.g. read from a reference checkpoint) into an
    ``[out, in]`` parameter or ``torch.nn.Linear`` of this framework."""
    lp = LinearParams(weight_in_out.shape[0], weight_in_out.shape[1], bias is not None, dtype=weight_in_out.dtype)
    with torch.no_grad():
        lp.weight.copy_(weight_in_out)
        if bias is not None:
            lp.bias.copy_(bias)
    lp.load_into(target)
