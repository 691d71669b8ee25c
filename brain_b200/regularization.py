"""Regularisation (crates/brain-regularization/src/): weight penalties (L1 / L2 / elastic net,
decoupled decay), dropout family (standard, alpha, spatial, DropConnect, DropPath / stochastic depth,
Monte-Carlo dropout), label smoothing, mixup / cutmix / cutout augmentation, gradient-noise
perturbation, elastic weight consolidation, curriculum pacing and early stopping."""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .nn.module import Module


def l1_penalty(params, weight: float) -> torch.Tensor:
    return weight * sum(p.abs().sum() for p in params)


def l2_penalty(params, weight: float) -> torch.Tensor:
    return 0.5 * weight * sum(p.pow(2).sum() for p in params)


def elastic_net_penalty(params, l1: float, l2: float) -> torch.Tensor:
    return l1_penalty(params, l1) + l2_penalty(params, l2)


@torch.no_grad()
def decoupled_weight_decay_(params, lr: float, wd: float) -> None:
    for p in params:
        p.mul_(1 - lr * wd)


class Dropout(Module):
    def __init__(self, p=0.1):
        super().__init__()
        self.p = p

    def forward(self, x):
        return F.dropout(x, self.p, self.training)


class AlphaDropout(Dropout):
    def forward(self, x):
        return F.alpha_dropout(x, self.p, self.training)


class Dropout2d(Dropout):
    def forward(self, x):
        return F.dropout2d(x, self.p, self.training)


class DropPath(Dropout):
    """Stochastic depth: drop the whole residual branch per sample."""

    def forward(self, x):
        if not self.training or self.p == 0.0:
            return x
        keep = 1 - self.p
        mask = x.new_empty((x.shape[0],) + (1,) * (x.dim() - 1)).bernoulli_(keep)
        return x * mask / keep


class DropConnect(Module):
    """Randomly zero weights of a wrapped linear layer during training."""

    def __init__(self, linear: torch.nn.Module, p=0.1):
        super().__init__()
        self.linear, self.p = linear, p

    def forward(self, x):
        w = self.linear.weight
        if self.training and self.p > 0:
            w = F.dropout(w, self.p, True)
        return F.linear(x, w, getattr(self.linear, "bias", None))


def mc_dropout_predict(model: torch.nn.Module, x, samples: int = 20):
    """Monte-Carlo dropout: mean and variance of predictions with dropout active."""
    was = model.training
    model.train()
    with torch.no_grad():
        outs = torch.stack([model(x).float() for _ in range(samples)])
    model.train(was)
    return outs.mean(0), outs.var(0)


def smooth_labels(target: torch.Tensor, num_classes: int, eps: float = 0.1) -> torch.Tensor:
    oh = F.one_hot(target, num_classes).float()
    return oh * (1 - eps) + eps / num_classes


def mixup(x, y_onehot, alpha=0.2, generator=None):
    lam = float(torch.distributions.Beta(alpha, alpha).sample()) if alpha > 0 else 1.0
    perm = torch.randperm(x.shape[0], generator=generator).to(x.device)
    return lam * x + (1 - lam) * x[perm], lam * y_onehot + (1 - lam) * y_onehot[perm]


def cutmix(x, y_onehot, alpha=1.0, generator=None):
    lam = float(torch.distributions.Beta(alpha, alpha).sample())
    B, _, H, W = x.shape
    perm = torch.randperm(B, generator=generator).to(x.device)
    rh, rw = int(H * math.sqrt(1 - lam)), int(W * math.sqrt(1 - lam))
    cy, cx = torch.randint(H, (1,), generator=generator).item(), torch.randint(W, (1,), generator=generator).item()
    y0, y1, x0, x1 = max(cy - rh // 2, 0), min(cy + rh // 2, H), max(cx - rw // 2, 0), min(cx + rw // 2, W)
    x = x.clone()
    x[:, :, y0:y1, x0:x1] = x[perm, :, y0:y1, x0:x1]
    lam = 1 - (y1 - y0) * (x1 - x0) / (H * W)
    return x, lam * y_onehot + (1 - lam) * y_onehot[perm]


def cutout(x, size=8, generator=None):
    B, _, H, W = x.shape
    x = x.clone()
    for b in range(B):
        cy = torch.randint(H, (1,), generator=generator).item()
        cx = torch.randint(W, (1,), generator=generator).item()
        x[b, :, max(cy - size // 2, 0):cy + size // 2, max(cx - size // 2, 0):cx + size // 2] = 0
    return x


@torch.no_grad()
def add_gradient_noise_(params, std: float, generator=None) -> None:
    for p in params:
        if p.grad is not None:
            p.grad.add_(torch.randn(p.grad.shape, generator=generator).to(p.grad) * std)


class EWC:
    """Elastic weight consolidation: F_i (theta_i - theta*_i)^2 penalty from a diagonal Fisher."""

    def __init__(self, model: torch.nn.Module, fisher: dict, lam: float = 1.0):
        self.anchor = {n: p.detach().clone() for n, p in model.named_parameters()}
        self.fisher, self.lam = fisher, lam

    @staticmethod
    def diagonal_fisher(model, batches, loss_fn) -> dict:
        fisher = {n: torch.zeros_like(p) for n, p in model.named_parameters()}
        for x, y in batches:
            model.zero_grad()
            loss_fn(model(x), y).backward()
            for n, p in model.named_parameters():
                if p.grad is not None:
                    fisher[n] += p.grad.detach() ** 2 / len(batches)
        return fisher

    def penalty(self, model) -> torch.Tensor:
        return self.lam / 2 * sum((self.fisher[n] * (p - self.anchor[n]) ** 2).sum()
                                  for n, p in model.named_parameters() if n in self.fisher)


class CurriculumScheduler:
    """Fraction of the (difficulty-sorted) data available at a step: linear / root / geometric pacing."""

    def __init__(self, total_steps: int, start_frac=0.2, kind="linear"):
        self.total, self.start, self.kind = total_steps, start_frac, kind

    def fraction(self, step: int) -> float:
        t = min(1.0, step / max(1, self.total))
        if self.kind == "root":
            return min(1.0, math.sqrt(self.start ** 2 + (1 - self.start ** 2) * t))
        if self.kind == "geometric":
            return min(1.0, self.start * (1 / self.start) ** t)
        return min(1.0, self.start + (1 - self.start) * t)


class EarlyStopper:
    def __init__(self, patience=5, min_delta=0.0, mode="min"):
        self.patience, self.min_delta, self.mode = patience, min_delta, mode
        self.best, self.bad = None, 0

    def step(self, metric: float) -> bool:
        better = self.best is None or (metric < self.best - self.min_delta if self.mode == "min"
                                       else metric > self.best + self.min_delta)
        if better:
            self.best, self.bad = metric, 0
        else:
            self.bad += 1
        return self.bad >= self.patience


# The reference's spellings (crates/brain-regularization/src: label_smooth.rs smooth_targets, augment.rs
# apply_mixup / apply_cutout_2d, ewc.rs ElasticWeightConsolidation, regularizers.rs ElasticNetRegularizer,
# normalization/{batch,group}.rs BatchNorm1d / InstanceNorm1d).
smooth_targets = smooth_labels
apply_mixup = mixup
apply_cutout_2d = cutout
ElasticWeightConsolidation = EWC


class ElasticNetRegularizer:
    """alpha * (l1_ratio * sum|w| + (1 - l1_ratio) / 2 * sum w^2) over the given parameters."""

    def __init__(self, alpha: float = 1e-4, l1_ratio: float = 0.5):
        self.alpha, self.l1_ratio = alpha, l1_ratio

    def penalty(self, params) -> torch.Tensor:
        params = list(params)
        l1 = sum(p.abs().sum() for p in params)
        l2 = sum((p * p).sum() for p in params)
        return self.alpha * (self.l1_ratio * l1 + (1 - self.l1_ratio) * 0.5 * l2)

    __call__ = penalty


from .nn.layers import BatchNorm1d, InstanceNorm1d  # noqa: E402,F401
