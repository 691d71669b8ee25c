"""Quantisation workflow pieces: KL-divergence (entropy) calibration, static and dynamic quantisers,
requantisation, error analysis, per-layer mixed precision, a quantised Conv2d, structured pruning with
iterative and lottery-ticket schedules, whole-model graph quantisation and a small benchmark.

Reference: crates/brain-quantization/src/calibration.rs (EntropyObserver), quant_static.rs
(StaticQuantizer), quant_dynamic.rs (DynamicQuantizer), ops.rs (requantize, requantize_per_channel),
error_analysis.rs (analyze_quantization_error), mixed.rs (MixedPrecisionQuantizer), qconv.rs (QConv2d),
prune/mod.rs (StructuredPruner, IterativePruneSchedule, LotteryTicketSchedule), graph_quant.rs
(GraphQuantizer), bench_quant.rs (QuantBench).

Integer GEMMs go through ``int8_matmul`` (``torch._int_mm``: int8 x int8 -> int32 with exact
accumulation, on the int8 tensor-core path of cuBLASLt on a GPU) whenever the shapes allow it.
"""
from __future__ import annotations

import copy
import math
import time
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import QLinear, QuantDType, QuantScheme, dequantize_tensor, quantize_tensor


# ------------------------------------------------------------------------------------------ integer GEMM
def int8_matmul(a_q: torch.Tensor, b_q: torch.Tensor) -> torch.Tensor:
    """int32 [M, N] = a_q [M, K] @ b_q [N, K]^T, exact. Uses torch._int_mm when M > 16 and K, N are
    multiples of 8, else an int64 matmul (CPU) / float matmul of integers (exact below 2^24)."""
    M, K = a_q.shape
    N = b_q.shape[0]
    if M > 16 and K % 8 == 0 and N % 8 == 0:
        return torch._int_mm(a_q.contiguous(), b_q.t().contiguous())
    if a_q.is_cuda:
        return (a_q.float() @ b_q.float().t()).round().to(torch.int32)
    return (a_q.to(torch.int64) @ b_q.to(torch.int64).t()).to(torch.int32)


def requantize(acc: torch.Tensor, in_scale: float, w_scale, out_scale: float, out_zp: int = 0,
               dtype: QuantDType = QuantDType.INT8) -> torch.Tensor:
    """int32 accumulators -> output integers: round(acc in_scale w_scale / out_scale) + zp, clamped.
    ``w_scale`` may be a per-output-channel vector (per-channel requantisation)."""
    qmin, qmax = dtype.qrange()
    ws = torch.as_tensor(w_scale, dtype=torch.float64, device=acc.device)
    m = (in_scale * ws / out_scale)
    y = torch.round(acc.double() * (m.reshape(1, -1) if ws.dim() else m)) + out_zp
    return y.clamp(qmin, qmax).to(torch.int8 if dtype.bits <= 8 and qmin < 0 else torch.int32)


def requantize_per_channel(acc, in_scale, w_scales, out_scale, out_zp=0, dtype=QuantDType.INT8):
    return requantize(acc, in_scale, w_scales, out_scale, out_zp, dtype)


# ------------------------------------------------------------------------------------------ calibration
class EntropyObserver:
    """KL-divergence calibration (the TensorRT entropy method): a |x| histogram of ``bins`` bins is built
    with ``torch.histc`` on the input's device and accumulated on the host; the clipping threshold is the bin edge whose 128-level quantised
    distribution has the smallest KL divergence to the clipped reference distribution."""

    def __init__(self, bins: int = 2048, levels: int = 128):
        self.bins, self.levels = bins, levels
        self.hist = None
        self.max = 0.0

    def observe(self, x: torch.Tensor) -> None:
        a = x.detach().abs().float().reshape(-1)
        m = float(a.max()) if a.numel() else 0.0
        if self.hist is None:
            self.max = max(m, 1e-12)
            self.hist = torch.histc(a, self.bins, 0, self.max).double().cpu()
            return
        if m > self.max:  # re-bin the old histogram onto the wider range
            old_edges = torch.linspace(0, self.max, self.bins + 1, dtype=torch.float64)[:-1] + self.max / self.bins / 2
            self.max = m
            idx = (old_edges / self.max * self.bins).long().clamp(max=self.bins - 1)
            h = torch.zeros(self.bins, dtype=torch.float64).index_add_(0, idx, self.hist)
            self.hist = h
        self.hist += torch.histc(a, self.bins, 0, self.max).double().cpu()

    def threshold(self) -> float:
        h = self.hist
        best_kl, best_i = math.inf, self.bins
        for i in range(self.levels, self.bins + 1):
            ref = h[:i].clone()
            ref[-1] += h[i:].sum()  # clip the tail into the last bin
            # quantise the first i bins into `levels` groups, spread each group's mass over its nonzero bins
            grp = torch.div(torch.arange(i) * self.levels, i, rounding_mode="floor")
            nz = (h[:i] > 0).double()
            gsum = torch.zeros(self.levels, dtype=torch.float64).index_add_(0, grp, h[:i])
            gcnt = torch.zeros(self.levels, dtype=torch.float64).index_add_(0, grp, nz)
            q = torch.where(nz > 0, gsum[grp] / gcnt[grp].clamp_min(1), torch.zeros_like(nz))
            p, qq = ref / ref.sum().clamp_min(1e-300), q / q.sum().clamp_min(1e-300)
            mask = p > 0
            qq = torch.where(mask & (qq == 0), torch.full_like(qq, 1e-8), qq)  # smooth empty quantised bins
            kl = float((p[mask] * torch.log(p[mask] / qq[mask])).sum())
            if kl < best_kl:
                best_kl, best_i = kl, i
        return (best_i + 0.5) * self.max / self.bins

    def scale_zp(self, dtype: QuantDType = QuantDType.INT8, symmetric: bool = True):
        return self.threshold() / dtype.qrange()[1], 0


# ------------------------------------------------------------------------------------------ quantisers
@dataclass
class QuantErrorReport:
    mse: float
    max_abs_error: float
    sqnr_db: float
    relative_error: float


def analyze_quantization_error(x: torch.Tensor, x_hat: torch.Tensor) -> QuantErrorReport:
    """MSE, worst absolute error, signal-to-quantisation-noise ratio (dB) and relative Frobenius error."""
    x, x_hat = x.double(), x_hat.double()
    e = x - x_hat
    ps, pn = float((x * x).mean()), float((e * e).mean())
    return QuantErrorReport(pn, float(e.abs().max()), 10 * math.log10(ps / pn) if pn > 0 else math.inf,
                            float(e.norm() / x.norm().clamp_min(1e-300)))


class DynamicQuantizer:
    """Per-row (per-token) symmetric int8 activations computed at run time, int8 weights per output
    channel, int32 accumulation and float rescale: y = (xq W_q^T) s_x s_w + b."""

    def __init__(self, linear: nn.Linear):
        w = linear.weight.detach().float()
        q, s, _ = quantize_tensor(w, QuantDType.INT8, True, QuantScheme.PER_CHANNEL, axis=0)
        self.w_q, self.w_s = q.reshape(w.shape), s.reshape(-1)
        self.bias = None if linear.bias is None else linear.bias.detach().float()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1]).float()
        xs = x2.abs().amax(1).clamp_min(1e-12) / 127.0
        xq = torch.round(x2 / xs[:, None]).clamp(-127, 127).to(torch.int8)
        y = int8_matmul(xq, self.w_q.to(xq.device)).float() * xs[:, None] * self.w_s.to(x.device)[None, :]
        if self.bias is not None:
            y = y + self.bias.to(x.device)
        return y.reshape(*x.shape[:-1], -1).to(x.dtype)


class StaticQuantizer:
    """Calibrated activation scale (min-max, percentile or entropy observer fed by ``calibrate``), fixed at
    inference: y = (round(x / s_x) W_q^T) s_x s_w + b."""

    def __init__(self, linear: nn.Linear, observer=None):
        from . import MinMaxObserver
        self.dyn = DynamicQuantizer(linear)
        self.obs = observer or MinMaxObserver()
        self.x_scale = None

    def calibrate(self, x: torch.Tensor) -> None:
        self.obs.observe(x)

    def freeze(self) -> float:
        self.x_scale = float(self.obs.scale_zp(QuantDType.INT8, True)[0])
        return self.x_scale

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.x_scale is None:
            self.freeze()
        x2 = x.reshape(-1, x.shape[-1]).float()
        xq = torch.round(x2 / self.x_scale).clamp(-127, 127).to(torch.int8)
        d = self.dyn
        y = int8_matmul(xq, d.w_q.to(xq.device)).float() * self.x_scale * d.w_s.to(x.device)[None, :]
        if d.bias is not None:
            y = y + d.bias.to(x.device)
        return y.reshape(*x.shape[:-1], -1).to(x.dtype)


class MixedPrecisionQuantizer:
    """Chooses, per weight tensor, the fewest bits among ``candidates`` whose SQNR meets ``min_sqnr_db``
    (8 bits otherwise); returns {name: bits} and the quantised-dequantised weights."""

    def __init__(self, candidates=(4, 8), min_sqnr_db: float = 30.0, group_size: int = 64):
        self.cand, self.min_db, self.gs = sorted(candidates), min_sqnr_db, group_size

    def _roundtrip(self, w: torch.Tensor, bits: int) -> torch.Tensor:
        dt = QuantDType.INT4 if bits == 4 else QuantDType.INT8
        if w.numel() % self.gs == 0:
            q, s, _ = quantize_tensor(w.float(), dt, True, QuantScheme.GROUP_WISE, group_size=self.gs)
            return (q.float().reshape(-1, self.gs) * s.reshape(-1, 1)).reshape(w.shape)
        q, s, zp = quantize_tensor(w.float(), dt, True)
        return dequantize_tensor(q, s, zp, w.shape)

    def plan(self, named_weights) -> dict:
        out = {}
        for name, w in named_weights:
            out[name] = next((b for b in self.cand
                              if analyze_quantization_error(w, self._roundtrip(w, b)).sqnr_db >= self.min_db), 8)
        return out


class QConv2d(nn.Module):
    """Conv2d with int8 weights (per output channel) dequantised on the fly; optional dynamic int8
    activations through an im2col int8 GEMM (per-image-patch-row scales)."""

    def __init__(self, conv: nn.Conv2d, act_quant: bool = False):
        super().__init__()
        w = conv.weight.detach().float()
        q, s, _ = quantize_tensor(w, QuantDType.INT8, True, QuantScheme.PER_CHANNEL, axis=0)
        self.register_buffer("w_q", q.reshape(w.shape))
        self.register_buffer("w_s", s.reshape(-1))
        self.register_buffer("bias", None if conv.bias is None else conv.bias.detach().float())
        self.stride, self.padding, self.dilation, self.groups = conv.stride, conv.padding, conv.dilation, conv.groups
        self.act_quant = act_quant and conv.groups == 1

    def weight(self) -> torch.Tensor:
        return self.w_q.float() * self.w_s.view(-1, 1, 1, 1)

    def forward(self, x):
        if not self.act_quant:
            return F.conv2d(x.float(), self.weight(), self.bias, self.stride, self.padding, self.dilation,
                            self.groups).to(x.dtype)
        B, C, H, W = x.shape
        O, _, kh, kw = self.w_q.shape
        cols = F.unfold(x.float(), (kh, kw), self.dilation, self.padding, self.stride)  # [B, C kh kw, L]
        L = cols.shape[-1]
        a = cols.transpose(1, 2).reshape(B * L, -1)
        xs = a.abs().amax(1).clamp_min(1e-12) / 127.0
        aq = torch.round(a / xs[:, None]).clamp(-127, 127).to(torch.int8)
        y = int8_matmul(aq, self.w_q.reshape(O, -1)).float() * xs[:, None] * self.w_s[None, :]
        if self.bias is not None:
            y = y + self.bias
        Ho = (H + 2 * self.padding[0] - self.dilation[0] * (kh - 1) - 1) // self.stride[0] + 1
        Wo = (W + 2 * self.padding[1] - self.dilation[1] * (kw - 1) - 1) // self.stride[1] + 1
        return y.reshape(B, Ho, Wo, O).permute(0, 3, 1, 2).to(x.dtype)


# ------------------------------------------------------------------------------------------ pruning
class StructuredPruner:
    """Zeroes whole output channels (rows) with the smallest L2 norms; returns the kept-row mask."""

    def __init__(self, sparsity: float):
        self.sparsity = sparsity

    @torch.no_grad()
    def prune_(self, w: torch.Tensor) -> torch.Tensor:
        norms = w.reshape(w.shape[0], -1).float().norm(dim=1)
        k = int(round(self.sparsity * w.shape[0]))
        keep = torch.ones(w.shape[0], dtype=torch.bool, device=w.device)
        if k > 0:
            keep[torch.argsort(norms, stable=True)[:k]] = False
        w[~keep] = 0
        return keep


class IterativePruneSchedule:
    """Gradual magnitude pruning (Zhu and Gupta 2017): s_t = s_f + (s_i - s_f) (1 - (t - t0) / (n dt))^3
    between step t0 and t0 + n dt, pruning every dt steps."""

    def __init__(self, initial_sparsity: float = 0.0, final_sparsity: float = 0.9, begin_step: int = 0,
                 end_step: int = 1000, frequency: int = 100):
        self.si, self.sf, self.t0, self.t1, self.dt = initial_sparsity, final_sparsity, begin_step, end_step, frequency

    def sparsity_at(self, step: int) -> float:
        if step <= self.t0:
            return self.si
        if step >= self.t1:
            return self.sf
        frac = (step - self.t0) / (self.t1 - self.t0)
        return self.sf + (self.si - self.sf) * (1.0 - frac) ** 3

    def should_prune(self, step: int) -> bool:
        return self.t0 <= step <= self.t1 and (step - self.t0) % self.dt == 0


class LotteryTicketSchedule:
    """Iterative magnitude pruning with rewinding (Frankle and Carbin 2019): after each round keep the
    largest (1 - rate) of the surviving weights and reset the survivors to their initial values."""

    def __init__(self, model: nn.Module, rate_per_round: float = 0.2):
        self.init = copy.deepcopy({k: v.detach().clone() for k, v in model.state_dict().items()})
        self.masks = {n: torch.ones_like(p, dtype=torch.bool) for n, p in model.named_parameters() if p.dim() > 1}
        self.rate, self.round = rate_per_round, 0

    @torch.no_grad()
    def next_round(self, model: nn.Module) -> float:
        params = dict(model.named_parameters())
        for n, m in self.masks.items():
            alive = params[n].detach().abs()[m]
            k = int(self.rate * alive.numel())
            if k > 0:
                thr = torch.kthvalue(alive.float().cpu(), k).values.item()
                m &= params[n].detach().abs() > thr
        model.load_state_dict(self.init)
        for n, m in self.masks.items():
            params[n].mul_(m)
        self.round += 1
        tot = sum(m.numel() for m in self.masks.values())
        return 1.0 - sum(int(m.sum()) for m in self.masks.values()) / max(tot, 1)


# ------------------------------------------------------------------------------------------ model-level
class GraphQuantizer:
    """Replaces every nn.Linear (and optionally nn.Conv2d) of a model by its int8 counterpart, skipping
    modules whose qualified names are in ``skip``; returns the list of replaced names."""

    def __init__(self, act_quant: bool = False, convs: bool = True, skip=()):
        self.act_quant, self.convs, self.skip = act_quant, convs, set(skip)

    def quantize_(self, model: nn.Module) -> list[str]:
        done = []
        for name, mod in list(model.named_modules()):
            for cname, child in list(mod.named_children()):
                full = f"{name}.{cname}" if name else cname
                if full in self.skip:
                    continue
                if isinstance(child, nn.Linear):
                    setattr(mod, cname, QLinear(child, self.act_quant))
                    done.append(full)
                elif self.convs and isinstance(child, nn.Conv2d):
                    setattr(mod, cname, QConv2d(child, self.act_quant))
                    done.append(full)
        return done


@dataclass
class QuantBenchReport:
    float_ms: float
    quant_ms: float
    speedup: float
    max_abs_diff: float
    weight_bytes_float: int
    weight_bytes_quant: int


def quant_bench(float_fn, quant_fn, x: torch.Tensor, iters: int = 10, weight_bytes=(0, 0)) -> QuantBenchReport:
    """Times a float and a quantised callable on the same input (CUDA events on a GPU, wall clock on the
    CPU, after one warm-up call each) and reports the largest output difference."""
    def run(fn):
        fn(x)
        if x.is_cuda:
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(iters):
                y = fn(x)
            e.record()
            torch.cuda.synchronize()
            return s.elapsed_time(e) / iters, y
        t0 = time.perf_counter()
        for _ in range(iters):
            y = fn(x)
        return (time.perf_counter() - t0) * 1e3 / iters, y
    tf, yf = run(float_fn)
    tq, yq = run(quant_fn)
    return QuantBenchReport(tf, tq, tf / tq if tq > 0 else math.inf, float((yf.float() - yq.float()).abs().max()),
                            weight_bytes[0], weight_bytes[1])
