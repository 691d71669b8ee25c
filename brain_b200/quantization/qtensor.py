"""Quantised-tensor objects with the reference's names: ``QParams`` / ``QuantTensor`` (integer data plus
its scale and zero point, per tensor or per channel), ``AffineQuantizer`` / ``SymmetricQuantizer``,
``ActQuantizer`` with dynamic per-token int8 quantisation, ``MagnitudePruner`` returning a
``PruneResult``, float16 / bfloat16 conversions and int4 buffer packing.

Reference: crates/brain-quantization/src/core.rs (QParams, QuantTensor), quantizer.rs (affine and
symmetric quantizers), act_quant.rs (ActQuantizer, quantize_per_token), prune/mod.rs (MagnitudePruner,
PruneResult), dtype_map.rs (f16 / bf16 conversions), helper.rs (pack_i8_to_i4_buffer), utils.rs
(compute_scale_zero_point, quantize_val, dequantize_val, minmax, percentile_slice).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import QuantDType, pack_int4, unpack_int4


def compute_scale_zero_point(lo: float, hi: float, qmin: int, qmax: int, symmetric: bool = False):
    """(scale, zero_point) mapping [lo, hi] (widened to include 0) onto [qmin, qmax]."""
    lo, hi = min(lo, 0.0), max(hi, 0.0)
    if symmetric:
        amax = max(abs(lo), abs(hi), 1e-12)
        return amax / qmax, 0
    scale = max((hi - lo) / (qmax - qmin), 1e-12)
    return scale, int(round(qmin - lo / scale))


def quantize_val(x: float, scale: float, zp: int, qmin: int, qmax: int) -> int:
    return int(min(max(round(x / scale + zp), qmin), qmax))


def dequantize_val(q: int, scale: float, zp: int) -> float:
    return (q - zp) * scale


def minmax(x: torch.Tensor) -> tuple[float, float]:
    return float(x.min()), float(x.max())


def percentile_slice(x: torch.Tensor, pct: float) -> float:
    return float(torch.quantile(x.float().reshape(-1), pct / 100.0))


@dataclass
class QParams:
    scale: torch.Tensor       # [] or [C]
    zero_point: torch.Tensor  # same shape as scale
    dtype: QuantDType = QuantDType.INT8
    axis: int | None = None   # channel axis for per-channel parameters

    def _bcast(self, t, ndim):
        if self.axis is None:
            return t
        shape = [1] * ndim
        shape[self.axis] = -1
        return t.reshape(shape)


@dataclass
class QuantTensor:
    data: torch.Tensor
    qparams: QParams

    @classmethod
    def from_float(cls, x: torch.Tensor, dtype: QuantDType = QuantDType.INT8, symmetric: bool = True,
                   axis: int | None = None) -> "QuantTensor":
        return (SymmetricQuantizer(dtype, axis) if symmetric else AffineQuantizer(dtype, axis)).quantize(x)

    def dequantize(self) -> torch.Tensor:
        p = self.qparams
        s, z = p._bcast(p.scale, self.data.dim()), p._bcast(p.zero_point, self.data.dim())
        return (self.data.float() - z) * s

    @property
    def shape(self):
        return tuple(self.data.shape)

    def nbytes(self) -> int:
        bits = self.qparams.dtype.bits
        return (self.data.numel() * bits + 7) // 8


class AffineQuantizer:
    """Asymmetric min/max quantisation, per tensor or per channel (``axis``)."""

    symmetric = False

    def __init__(self, dtype: QuantDType = QuantDType.UINT8, axis: int | None = None):
        self.dtype, self.axis = dtype, axis

    def fit(self, x: torch.Tensor) -> QParams:
        qmin, qmax = self.dtype.qrange()
        xf = x.float()
        if self.axis is None:
            lo, hi = xf.min().clamp_max(0), xf.max().clamp_min(0)
        else:
            red = [d for d in range(x.dim()) if d != self.axis]
            lo, hi = xf.amin(red).clamp_max(0), xf.amax(red).clamp_min(0)
        if self.symmetric:
            scale = torch.maximum(lo.abs(), hi.abs()).clamp_min(1e-12) / qmax
            zp = torch.zeros_like(scale)
        else:
            scale = ((hi - lo) / (qmax - qmin)).clamp_min(1e-12)
            zp = torch.round(qmin - lo / scale)
        return QParams(scale, zp, self.dtype, self.axis)

    def quantize(self, x: torch.Tensor, qparams: QParams | None = None) -> QuantTensor:
        p = qparams or self.fit(x)
        qmin, qmax = self.dtype.qrange()
        s, z = p._bcast(p.scale, x.dim()), p._bcast(p.zero_point, x.dim())
        q = torch.clamp(torch.round(x.float() / s + z), qmin, qmax)
        store = torch.int32 if self.dtype.bits > 8 else (torch.int8 if qmin < 0 else torch.uint8)
        return QuantTensor(q.to(store), p)

    def dequantize(self, qt: QuantTensor) -> torch.Tensor:
        return qt.dequantize()


class SymmetricQuantizer(AffineQuantizer):
    """Zero point 0, scale = amax / qmax (per tensor or per channel)."""

    symmetric = True

    def __init__(self, dtype: QuantDType = QuantDType.INT8, axis: int | None = None):
        super().__init__(dtype, axis)


def quantize_per_token(x: torch.Tensor):
    """Dynamic symmetric int8 per row of the last dimension: (q int8 [..., D], scale f32 [..., 1])."""
    xf = x.float()
    scale = xf.abs().amax(-1, keepdim=True).clamp_min(1e-12) / 127.0
    return torch.clamp(torch.round(xf / scale), -127, 127).to(torch.int8), scale


class ActQuantizer:
    """Activation quantiser: ``mode="per_token"`` (dynamic, one scale per token) or ``"per_tensor"``
    with a calibrated running amax (``observe`` then ``quantize``)."""

    def __init__(self, mode: str = "per_token", momentum: float = 0.9):
        self.mode, self.momentum, self.amax = mode, momentum, None

    def observe(self, x: torch.Tensor) -> None:
        a = float(x.abs().max())
        self.amax = a if self.amax is None else self.momentum * self.amax + (1 - self.momentum) * a

    def quantize(self, x: torch.Tensor):
        if self.mode == "per_token":
            return quantize_per_token(x)
        amax = self.amax if self.amax is not None else float(x.abs().max())
        scale = torch.tensor(max(amax, 1e-12) / 127.0)
        return torch.clamp(torch.round(x.float() / scale), -127, 127).to(torch.int8), scale


@dataclass
class PruneResult:
    mask: torch.Tensor
    sparsity: float
    threshold: float


class MagnitudePruner:
    """Zero the smallest-magnitude fraction of a tensor (global over the tensor, or per output row with
    ``per_row``); returns the mask, achieved sparsity and threshold."""

    def __init__(self, sparsity: float, per_row: bool = False):
        if not 0.0 <= sparsity < 1.0:
            raise ValueError("sparsity must be in [0, 1)")
        self.sparsity, self.per_row = sparsity, per_row

    def prune(self, w: torch.Tensor, in_place: bool = True) -> PruneResult:
        a = w.detach().abs().float()
        if self.per_row and w.dim() > 1:
            flat = a.reshape(w.shape[0], -1)
            k = int(self.sparsity * flat.shape[1])
            thr = flat.kthvalue(k, dim=1, keepdim=True).values if k > 0 else flat.new_full((flat.shape[0], 1), -1.0)
            mask = (flat > thr).reshape(w.shape)
            t = float(thr.max())
        else:
            k = int(self.sparsity * a.numel())
            t = float(a.reshape(-1).kthvalue(k).values) if k > 0 else -1.0
            mask = a > t
        if in_place:
            with torch.no_grad():
                w.mul_(mask.to(w.dtype))
        return PruneResult(mask, 1.0 - float(mask.float().mean()), t)


def f64_to_f16(x) -> torch.Tensor:
    return torch.as_tensor(x, dtype=torch.float64).to(torch.float16)


def f16_to_f64(x) -> torch.Tensor:
    return torch.as_tensor(x).to(torch.float64)


def f64_to_bf16(x) -> torch.Tensor:
    return torch.as_tensor(x, dtype=torch.float64).to(torch.bfloat16)


def bf16_to_f64(x) -> torch.Tensor:
    return torch.as_tensor(x).to(torch.float64)


def pack_i8_to_i4_buffer(q: torch.Tensor) -> torch.Tensor:
    """Signed values in [-8, 7], two per byte, low nibble first."""
    return pack_int4(q)


def unpack_i4_to_i8_buffer(p: torch.Tensor, numel: int) -> torch.Tensor:
    return unpack_int4(p, numel)
