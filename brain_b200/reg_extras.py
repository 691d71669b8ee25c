"""Regularisation extras: concrete (learnable-rate) dropout, Gaussian noise injection, FGSM perturbation,
consistency loss, Monte-Carlo dropout statistics, stop policies, a streaming Welford accumulator,
weight/spectral normalisation wrappers, a regulariser registry and a weighted regulariser stack.

Reference: crates/brain-regularization/src/dropout/adaptive.rs (ConcreteDropout), perturb.rs
(GaussianNoise, apply_fgsm_perturbation), consistency.rs (compute_consistency_loss),
dropout_uncertainty.rs (compute_mc_dropout_statistics), stopping.rs (StopOnBudget, StopOnPlateau,
StopAction), utils.rs (WelfordAccumulator), normalization/ (WeightNorm, SpectralNorm), registry.rs
(RegRegistry.parse_kind), regularizers.rs (WeightedRegularizer, RegStack).

``ConcreteDropout`` keeps its drop-rate logit as a trainable parameter (Gal et al. 2017): the relaxed
Bernoulli mask is differentiable, so the rate is learned with the network; the reference holds the
logit as a constant.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .regularization import elastic_net_penalty, l1_penalty, l2_penalty


class ConcreteDropout(nn.Module):
    """Relaxed-Bernoulli dropout with a learnable rate p = sigmoid(logit_p): for u ~ U(eps, 1 - eps), the
    relaxed drop indicator is z = sigmoid(clamp((logit_p + ln(u / (1 - u))) / temperature, -20, 20)) and
    y = x (1 - z) / (1 - p), unbiased in expectation (Gal et al. 2017; the reference multiplies by z
    itself, which keeps instead of drops with rate p); identity in eval. ``regularizer(weight_sq_sum,
    input_dim)`` is the concrete-dropout penalty weight_reg |W|^2 / (1 - p) - dropout_reg input_dim H(p)."""

    def __init__(self, initial_p: float = 0.1, temperature: float = 0.1, weight_regularizer: float = 1e-6,
                 dropout_regularizer: float = 1e-5):
        super().__init__()
        p = min(max(initial_p, 1e-4), 1 - 1e-4)
        self.logit_p = nn.Parameter(torch.tensor(math.log(p / (1 - p))))
        self.temperature = max(temperature, 1e-4)
        self.wr, self.dr = weight_regularizer, dropout_regularizer

    def current_p(self) -> float:
        return float(torch.sigmoid(self.logit_p.detach()))

    def forward(self, x, generator=None):
        if not self.training:
            return x
        eps = 1e-7
        u = torch.rand(x.shape, generator=generator, dtype=torch.float32).to(x.device).clamp(eps, 1 - eps)
        z = torch.sigmoid(((self.logit_p + torch.log(u / (1 - u))) / self.temperature).clamp(-20, 20))
        p = torch.sigmoid(self.logit_p)
        return x * (1 - z).to(x.dtype) / (1 - p)

    def regularizer(self, weight_sq_sum, input_dim: int):
        p = torch.sigmoid(self.logit_p)
        ent = -(p * torch.log(p) + (1 - p) * torch.log(1 - p))
        return self.wr * weight_sq_sum / (1 - p) - self.dr * input_dim * ent


class GaussianNoise(nn.Module):
    """x + N(0, std^2) in training (std clamped at 0), identity in eval."""

    def __init__(self, std_dev: float):
        super().__init__()
        self.std = max(std_dev, 0.0)

    def forward(self, x, generator=None):
        if not self.training or self.std == 0:
            return x
        return x + torch.randn(x.shape, generator=generator, dtype=torch.float32).to(x.device, x.dtype) * self.std

    inject = forward


def apply_fgsm_perturbation(x: torch.Tensor, grad: torch.Tensor, epsilon: float) -> torch.Tensor:
    """x + epsilon * sign(grad) (sign(0) = 0)."""
    if x.shape != grad.shape:
        raise ValueError(f"shape mismatch: {tuple(x.shape)} vs {tuple(grad.shape)}")
    return x + epsilon * torch.sign(grad)


def fgsm_example(model, loss_fn, x: torch.Tensor, target, epsilon: float) -> torch.Tensor:
    """The FGSM adversarial input for ``loss_fn(model(x), target)`` (one backward pass w.r.t. the input)."""
    xa = x.detach().clone().requires_grad_(True)
    loss = loss_fn(model(xa), target)
    g, = torch.autograd.grad(loss, xa)
    return apply_fgsm_perturbation(x.detach(), g, epsilon)


def compute_consistency_loss(pred1: torch.Tensor, pred2: torch.Tensor, weight: float = 1.0) -> torch.Tensor:
    """weight * mean squared difference of two predictions (e.g. two augmentations or student/teacher)."""
    if pred1.shape != pred2.shape:
        raise ValueError(f"shape mismatch: {tuple(pred1.shape)} vs {tuple(pred2.shape)}")
    return weight * ((pred1 - pred2) ** 2).mean()


@dataclass
class McDropoutResult:
    mean: torch.Tensor
    variance: torch.Tensor
    std_dev: torch.Tensor


def compute_mc_dropout_statistics(samples) -> McDropoutResult:
    """Per-element mean and population variance (clamped at 0) over stochastic forward passes
    (a list of same-shape tensors or one [S, ...] tensor)."""
    s = torch.stack(list(samples)) if not torch.is_tensor(samples) else samples
    if s.shape[0] == 0:
        raise ValueError("no samples")
    m = s.mean(0)
    v = ((s * s).mean(0) - m * m).clamp_min(0)
    return McDropoutResult(m, v, v.sqrt())


def mc_dropout_samples(model, x, num_samples: int = 30):
    """Run the model ``num_samples`` times with dropout active (train mode), other state untouched."""
    was = model.training
    model.train()
    with torch.no_grad():
        out = torch.stack([model(x) for _ in range(num_samples)])
    model.train(was)
    return out


class StopAction:
    HALT_TRAINING, REDUCE_LEARNING_RATE, WARN_ONLY = "halt", "reduce_lr", "warn"


class StopOnBudget:
    def __init__(self, max_steps: int):
        self.max_steps = max_steps

    def should_stop(self, step: int, loss: float) -> bool:
        return step >= self.max_steps


class StopOnPlateau:
    """Stop after ``patience`` consecutive losses that do not beat the best by more than min_loss_delta."""

    def __init__(self, patience: int, min_loss_delta: float = 0.0):
        self.patience, self.delta = patience, min_loss_delta
        self.best_loss, self.plateau_count = math.inf, 0

    def should_stop(self, step: int, loss: float) -> bool:
        if loss < self.best_loss - self.delta:
            self.best_loss, self.plateau_count = loss, 0
            return False
        self.plateau_count += 1
        return self.plateau_count >= self.patience


class WelfordAccumulator:
    """Streaming mean / variance (Welford 1962), element-wise over tensors of one shape; ``merge`` combines
    two accumulators (Chan et al.), so per-rank statistics can be reduced."""

    def __init__(self):
        self.n, self.mean, self.m2 = 0, None, None

    def update(self, x: torch.Tensor) -> None:
        x = x.double()
        self.n += 1
        if self.mean is None:
            self.mean, self.m2 = x.clone(), torch.zeros_like(x)
            return
        d = x - self.mean
        self.mean += d / self.n
        self.m2 += d * (x - self.mean)

    def merge(self, other: "WelfordAccumulator") -> None:
        if other.n == 0:
            return
        if self.n == 0:
            self.n, self.mean, self.m2 = other.n, other.mean.clone(), other.m2.clone()
            return
        n = self.n + other.n
        d = other.mean - self.mean
        self.mean = self.mean + d * other.n / n
        self.m2 = self.m2 + other.m2 + d * d * self.n * other.n / n
        self.n = n

    def variance(self, unbiased: bool = False) -> torch.Tensor:
        if self.n == 0:
            raise ValueError("empty accumulator")
        return self.m2 / (self.n - 1 if unbiased and self.n > 1 else self.n)


def weight_norm(module: nn.Module, name: str = "weight", dim: int = 0) -> nn.Module:
    """w = g v / |v| reparameterisation (Salimans and Kingma 2016) of ``module.<name>``."""
    return nn.utils.parametrizations.weight_norm(module, name, dim)


def spectral_norm(module: nn.Module, name: str = "weight", n_power_iterations: int = 1) -> nn.Module:
    """w / sigma_max(w) by power iteration on every forward in training."""
    return nn.utils.parametrizations.spectral_norm(module, name, n_power_iterations)


class RegKind:
    DROPOUT, ALPHA_DROPOUT, BATCH_NORM, LAYER_NORM, GROUP_NORM, INSTANCE_NORM = (
        "dropout", "alpha_dropout", "batch_norm", "layer_norm", "group_norm", "instance_norm")
    WEIGHT_NORM, SPECTRAL_NORM, L1, L2, ELASTIC_NET = "weight_norm", "spectral_norm", "l1", "l2", "elastic_net"


class RegRegistry:
    _NAMES = {"dropout": RegKind.DROPOUT, "alpha_dropout": RegKind.ALPHA_DROPOUT, "batch_norm": RegKind.BATCH_NORM,
              "batchnorm": RegKind.BATCH_NORM, "layer_norm": RegKind.LAYER_NORM, "layernorm": RegKind.LAYER_NORM,
              "group_norm": RegKind.GROUP_NORM, "groupnorm": RegKind.GROUP_NORM,
              "instance_norm": RegKind.INSTANCE_NORM, "instancenorm": RegKind.INSTANCE_NORM,
              "weight_norm": RegKind.WEIGHT_NORM, "weightnorm": RegKind.WEIGHT_NORM,
              "spectral_norm": RegKind.SPECTRAL_NORM, "spectralnorm": RegKind.SPECTRAL_NORM,
              "l1": RegKind.L1, "l2": RegKind.L2, "elastic_net": RegKind.ELASTIC_NET}

    @classmethod
    def parse_kind(cls, name: str) -> str:
        k = cls._NAMES.get(name.lower())
        if k is None:
            raise ValueError(f"Unknown regularization layer: {name}")
        return k


class WeightedRegularizer:
    """A weight penalty (l1, l2 or elastic_net with l1_ratio) scaled by ``weight``, over parameters."""

    def __init__(self, kind: str, weight: float, l1_ratio: float = 0.5):
        self.kind, self.weight, self.ratio = RegRegistry.parse_kind(kind), weight, l1_ratio

    def __call__(self, params) -> torch.Tensor:
        params = list(params)
        if self.kind == RegKind.L1:
            return l1_penalty(params, self.weight)
        if self.kind == RegKind.L2:
            return l2_penalty(params, self.weight)
        if self.kind == RegKind.ELASTIC_NET:
            return elastic_net_penalty(params, self.weight * self.ratio, self.weight * (1 - self.ratio))
        raise ValueError(f"{self.kind} is not a weight penalty")


class RegStack:
    """Sum of several weighted regularisers over the same parameters."""

    def __init__(self, regs=()):
        self.regs = list(regs)

    def add(self, reg: WeightedRegularizer) -> "RegStack":
        self.regs.append(reg)
        return self

    def __call__(self, params) -> torch.Tensor:
        params = list(params)
        return sum((r(params) for r in self.regs), torch.zeros(()))
