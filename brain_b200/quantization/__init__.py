"""Quantisation (crates/brain-quantization/src/): dtypes and schemes, group-wise int8 / int4
quantisation (``BlockQuantizer``, block_quant.rs:20-70; int4 packing, dtype_map.rs:88-95), quantised
linear layers with int32-style accumulation (``QLinear`` qlinear.rs:26-110, ``q8_matmul``
qmatmul.rs:34-66), calibration observers, SmoothQuant scales (act_quant.rs:47-74), fake quantisation
with a straight-through estimator, magnitude pruning, and the FP8 E4M3 **1x128 block-scaled** format
(declared but without math in the reference) used by the sm_100a FP8 GEMM (``csrc/fp8.cu``).
"""
from __future__ import annotations

import enum

import torch

from .fp8 import (dequantize_fp8_blockwise, fp8_linear, fp8_gemm_blockscaled, quantize_fp8_blockwise,  # noqa: F401
                  quantize_fp8_weight_blocks, quantize_fp8_rowwise, fp8_gemm_rowwise, fp8_linear_rowwise, Fp8Linear)


class QuantDType(enum.Enum):
    INT8 = "int8"
    UINT8 = "uint8"
    INT4 = "int4"
    UINT4 = "uint4"
    INT16 = "int16"
    UINT16 = "uint16"
    FP8E4M3 = "fp8e4m3"
    FP8E5M2 = "fp8e5m2"
    BF16 = "bf16"
    F16 = "f16"

    @property
    def bits(self) -> int:
        return {"int8": 8, "uint8": 8, "int4": 4, "uint4": 4, "int16": 16, "uint16": 16, "fp8e4m3": 8,
                "fp8e5m2": 8, "bf16": 16, "f16": 16}[self.value]

    def qrange(self) -> tuple[int, int]:
        b = self.bits
        if self.value.startswith("u"):
            return 0, 2 ** b - 1
        return -(2 ** (b - 1)), 2 ** (b - 1) - 1


class QuantScheme(enum.Enum):
    PER_TENSOR = "per_tensor"
    PER_CHANNEL = "per_channel"
    GROUP_WISE = "group_wise"


def quantize_tensor(x: torch.Tensor, dtype: QuantDType = QuantDType.INT8, symmetric: bool = True,
                    scheme: QuantScheme = QuantScheme.PER_TENSOR, axis: int = 0, group_size: int = 128):
    """Affine quantisation -> (q, scale, zero_point). Group-wise groups the last dimension."""
    qmin, qmax = dtype.qrange()
    xf = x.float()
    if scheme == QuantScheme.GROUP_WISE:
        xf = xf.reshape(-1, group_size)
        red = 1
    elif scheme == QuantScheme.PER_CHANNEL:
        xf = xf.movedim(axis, 0).reshape(x.shape[axis], -1)
        red = 1
    else:
        xf = xf.reshape(1, -1)
        red = 1
    if symmetric:
        amax = xf.abs().amax(red, keepdim=True).clamp_min(1e-12)
        scale = amax / qmax  # symmetric: +amax maps to qmax exactly (amax / 128 would clip it)
        zp = torch.zeros_like(scale)
    else:
        lo, hi = xf.amin(red, keepdim=True), xf.amax(red, keepdim=True)
        scale = ((hi - lo) / (qmax - qmin)).clamp_min(1e-12)
        zp = torch.round(qmin - lo / scale)
    q = torch.clamp(torch.round(xf / scale + zp), qmin, qmax)
    return q.to(torch.int32 if dtype.bits > 8 else torch.int8 if qmin < 0 else torch.uint8), scale, zp


def dequantize_tensor(q, scale, zp, shape=None, scheme: QuantScheme = QuantScheme.PER_TENSOR, axis: int = 0):
    x = (q.float() - zp) * scale
    if shape is None:
        return x
    if scheme == QuantScheme.PER_CHANNEL:
        moved = list(shape)
        moved.insert(0, moved.pop(axis))
        return x.reshape(moved).movedim(0, axis)
    return x.reshape(shape)


class BlockQuantizer:
    """Group-wise min/max quantisation of the last dimension (block_quant.rs:30-70)."""

    def __init__(self, block_size: int = 64, dtype: QuantDType = QuantDType.INT8, symmetric: bool = True):
        self.block, self.dtype, self.symmetric = block_size, dtype, symmetric

    def quantize_blocks(self, x: torch.Tensor):
        return quantize_tensor(x, self.dtype, self.symmetric, QuantScheme.GROUP_WISE, group_size=self.block)

    def dequantize_blocks(self, q, scale, zp, shape):
        return dequantize_tensor(q, scale, zp, shape, QuantScheme.GROUP_WISE)


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """Two signed 4-bit values per byte (low nibble first)."""
    u = (q.to(torch.int16).reshape(-1) & 0xF).to(torch.uint8)
    if u.numel() % 2:
        u = torch.cat([u, torch.zeros(1, dtype=torch.uint8, device=u.device)])
    return u[0::2] | (u[1::2] << 4)


def unpack_int4(p: torch.Tensor, numel: int) -> torch.Tensor:
    lo = (p & 0xF).to(torch.int16)
    hi = (p >> 4).to(torch.int16)
    v = torch.stack([lo, hi], 1).reshape(-1)[:numel]
    return torch.where(v > 7, v - 16, v).to(torch.int8)


def q8_matmul(a_q, a_scale, b_q, b_scale) -> torch.Tensor:
    """(a_q * a_scale) @ (b_q * b_scale)^T with exact integer accumulation (per-row scales)."""
    acc = a_q.to(torch.int64) @ b_q.to(torch.int64).t() if not a_q.is_cuda else (a_q.float() @ b_q.float().t())
    return acc.float() * a_scale.reshape(-1, 1).float() * b_scale.reshape(1, -1).float()


class QLinear(torch.nn.Module):
    """Weight-only or weight+activation int8 linear (per-output-channel weight scales)."""

    def __init__(self, linear: torch.nn.Module, act_quant: bool = False, group_size: int = 0):
        super().__init__()
        w = linear.weight.detach().float()
        self.out_features, self.in_features = w.shape
        self.group_size = group_size
        if group_size:
            q, s, _ = quantize_tensor(w, QuantDType.INT8, True, QuantScheme.GROUP_WISE, group_size=group_size)
        else:
            q, s, _ = quantize_tensor(w, QuantDType.INT8, True, QuantScheme.PER_CHANNEL, axis=0)
        self.register_buffer("w_q", q.reshape(w.shape))
        self.register_buffer("w_scale", s)
        b = getattr(linear, "bias", None)
        self.register_buffer("bias", None if b is None else b.detach().float())
        self.act_quant = act_quant

    def weight(self) -> torch.Tensor:
        if self.group_size:
            return (self.w_q.float().reshape(-1, self.group_size) * self.w_scale).reshape(self.w_q.shape)
        return self.w_q.float() * self.w_scale.reshape(-1, 1)

    def forward(self, x):
        if self.act_quant and not self.group_size:
            xq, xs, _ = quantize_tensor(x.reshape(-1, x.shape[-1]), QuantDType.INT8, True, QuantScheme.PER_CHANNEL,
                                        axis=0)
            y = q8_matmul(xq, xs, self.w_q, self.w_scale).reshape(*x.shape[:-1], self.out_features)
        else:
            y = x.float() @ self.weight().t()
        if self.bias is not None:
            y = y + self.bias
        return y.to(x.dtype)


class MinMaxObserver:
    def __init__(self):
        self.lo, self.hi = float("inf"), float("-inf")

    def observe(self, x):
        self.lo = min(self.lo, float(x.min()))
        self.hi = max(self.hi, float(x.max()))

    def scale_zp(self, dtype=QuantDType.INT8, symmetric=True):
        qmin, qmax = dtype.qrange()
        if symmetric:
            return max(abs(self.lo), abs(self.hi), 1e-12) / qmax, 0
        s = max(self.hi - self.lo, 1e-12) / (qmax - qmin)
        return s, round(qmin - self.lo / s)


class MovingAverageObserver(MinMaxObserver):
    def __init__(self, momentum=0.9):
        super().__init__()
        self.m = momentum

    def observe(self, x):
        lo, hi = float(x.min()), float(x.max())
        if self.lo == float("inf"):
            self.lo, self.hi = lo, hi
        else:
            self.lo = self.m * self.lo + (1 - self.m) * lo
            self.hi = self.m * self.hi + (1 - self.m) * hi


class PercentileObserver(MinMaxObserver):
    def __init__(self, pct=99.99):
        super().__init__()
        self.pct = pct
        self.samples = []

    def observe(self, x):
        self.samples.append(x.detach().float().flatten())
        allv = torch.cat(self.samples)
        k = max(1, int(allv.numel() * self.pct / 100))
        self.hi = float(allv.abs().kthvalue(k).values)
        self.lo = -self.hi


def smoothquant_scales(act_absmax: torch.Tensor, weight: torch.Tensor, alpha: float = 0.5) -> torch.Tensor:
    """Per-input-channel s = max|X|^alpha / max|W|^(1-alpha); use X/s and W*s."""
    w_absmax = weight.detach().float().abs().amax(0).clamp_min(1e-5)
    return (act_absmax.float().clamp_min(1e-5) ** alpha / w_absmax ** (1 - alpha)).clamp_min(1e-5)


class _FakeQuantSTE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, qmin, qmax):
        return torch.clamp(torch.round(x / scale), qmin, qmax) * scale

    @staticmethod
    def backward(ctx, g):
        return g, None, None, None


def fake_quantize(x, scale, dtype: QuantDType = QuantDType.INT8):
    qmin, qmax = dtype.qrange()
    return _FakeQuantSTE.apply(x, scale, qmin, qmax)


@torch.no_grad()
def magnitude_prune_(w: torch.Tensor, sparsity: float) -> torch.Tensor:
    """Zero the smallest |w| fraction in place; returns the keep mask."""
    k = int(w.numel() * sparsity)
    if k == 0:
        return torch.ones_like(w, dtype=torch.bool)
    thresh = w.abs().flatten().kthvalue(k).values
    mask = w.abs() > thresh
    w.mul_(mask)
    return mask


def to_csr(w: torch.Tensor):
    return w.to_sparse_csr()
