"""Loss functions (crates/brain-loss/src/): classification, regression, contrastive, adversarial,
segmentation, distillation and sequence losses, with a common ``Loss`` interface
(``forward(pred, target)``; reference ``Loss`` trait with ``forward_value``, core.rs:100).

Cross-entropy runs the fused sm_100a kernel on CUDA bf16 logits (``ops.cross_entropy``); the rest
are tensor-op compositions, differentiable through autograd.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import ops


def _reduce(x: torch.Tensor, reduction: str):
    if reduction == "mean":
        return x.mean()
    if reduction == "sum":
        return x.sum()
    return x


class Loss:
    reduction = "mean"

    def __call__(self, pred, target=None, *a, **kw):
        return self.forward(pred, target, *a, **kw)

    def forward(self, pred, target, *a, **kw):  # pragma: no cover - abstract
        raise NotImplementedError

    forward_value = forward


# ------------------------------------------------------------------ classification
class CrossEntropyLoss(Loss):
    """Softmax cross-entropy with label smoothing and ignore_index (classification/ce.rs:16-135)."""

    def __init__(self, label_smoothing: float = 0.0, ignore_index: int = -100, reduction: str = "mean",
                 weight: torch.Tensor | None = None):
        self.ls, self.ignore, self.reduction, self.weight = label_smoothing, ignore_index, reduction, weight

    def forward(self, logits, target):
        if self.weight is None:
            return ops.cross_entropy(logits, target, self.ignore, self.ls, self.reduction)
        return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), target.reshape(-1), self.weight,
                               ignore_index=self.ignore, label_smoothing=self.ls, reduction=self.reduction)

    forward_value_logits = forward


class NLLLoss(Loss):
    def __init__(self, reduction="mean", ignore_index=-100):
        self.reduction, self.ignore = reduction, ignore_index

    def forward(self, logp, target):
        return F.nll_loss(logp.float(), target, ignore_index=self.ignore, reduction=self.reduction)


class BCELoss(Loss):
    def __init__(self, reduction="mean", eps=1e-12):
        self.reduction, self.eps = reduction, eps

    def forward(self, p, t):
        p = p.float().clamp(self.eps, 1 - self.eps)
        return _reduce(-(t * p.log() + (1 - t) * (1 - p).log()), self.reduction)


class BCEWithLogitsLoss(Loss):
    def __init__(self, reduction="mean", pos_weight=None):
        self.reduction, self.pos_weight = reduction, pos_weight

    def forward(self, z, t):
        return F.binary_cross_entropy_with_logits(z.float(), t.float(), pos_weight=self.pos_weight,
                                                  reduction=self.reduction)


class FocalLoss(Loss):
    """Multi-class focal loss: -alpha (1 - p_t)^gamma log p_t (classification/focal.rs)."""

    def __init__(self, gamma=2.0, alpha=1.0, reduction="mean"):
        self.gamma, self.alpha, self.reduction = gamma, alpha, reduction

    def forward(self, logits, t):
        logp = F.log_softmax(logits.float(), -1).gather(-1, t[..., None]).squeeze(-1)
        p = logp.exp()
        return _reduce(-self.alpha * (1 - p) ** self.gamma * logp, self.reduction)


class HingeLoss(Loss):
    def __init__(self, margin=1.0, reduction="mean"):
        self.margin, self.reduction = margin, reduction

    def forward(self, scores, t):
        """Multi-class hinge (Crammer-Singer style) over logits and integer targets."""
        s = scores.float()
        correct = s.gather(-1, t[..., None])
        m = (self.margin + s - correct).clamp_min(0)
        m = m.scatter(-1, t[..., None], 0.0)
        return _reduce(m.sum(-1), self.reduction)


class KLDivLoss(Loss):
    def __init__(self, reduction="batchmean", log_target=False):
        self.reduction, self.log_target = reduction, log_target

    def forward(self, logp, target):
        return F.kl_div(logp.float(), target.float(), reduction=self.reduction, log_target=self.log_target)


class CTCLoss(Loss):
    def __init__(self, blank=0, reduction="mean"):
        self.blank, self.reduction = blank, reduction

    def forward(self, log_probs, targets, input_lengths, target_lengths):
        return F.ctc_loss(log_probs.float(), targets, input_lengths, target_lengths, self.blank, self.reduction)


# ------------------------------------------------------------------ regression
class MSELoss(Loss):
    def __init__(self, reduction="mean"):
        self.reduction = reduction

    def forward(self, p, t):
        return _reduce((p.float() - t.float()) ** 2, self.reduction)


class L1Loss(MSELoss):
    def forward(self, p, t):
        return _reduce((p.float() - t.float()).abs(), self.reduction)


class HuberLoss(Loss):
    def __init__(self, delta=1.0, reduction="mean"):
        self.delta, self.reduction = delta, reduction

    def forward(self, p, t):
        return F.huber_loss(p.float(), t.float(), reduction=self.reduction, delta=self.delta)


class SmoothL1Loss(HuberLoss):
    def forward(self, p, t):
        return F.smooth_l1_loss(p.float(), t.float(), reduction=self.reduction, beta=self.delta)


class LogCoshLoss(MSELoss):
    def forward(self, p, t):
        d = p.float() - t.float()
        return _reduce(d + F.softplus(-2 * d) - math.log(2.0), self.reduction)


class QuantileLoss(Loss):
    def __init__(self, q=0.5, reduction="mean"):
        self.q, self.reduction = q, reduction

    def forward(self, p, t):
        d = t.float() - p.float()
        return _reduce(torch.maximum(self.q * d, (self.q - 1) * d), self.reduction)


class PoissonNLLLoss(MSELoss):
    def forward(self, log_rate, t):
        return _reduce(log_rate.float().exp() - t.float() * log_rate.float(), self.reduction)


class GaussianNLLLoss(Loss):
    def __init__(self, eps=1e-6, reduction="mean"):
        self.eps, self.reduction = eps, reduction

    def forward(self, mu, t, var):
        v = var.float().clamp_min(self.eps)
        return _reduce(0.5 * (v.log() + (t.float() - mu.float()) ** 2 / v), self.reduction)


# ------------------------------------------------------------------ contrastive / metric learning
class CosineEmbeddingLoss(Loss):
    def __init__(self, margin=0.0, reduction="mean"):
        self.margin, self.reduction = margin, reduction

    def forward(self, x1, x2, y):
        return F.cosine_embedding_loss(x1.float(), x2.float(), y, self.margin, reduction=self.reduction)


class MarginRankingLoss(Loss):
    def __init__(self, margin=0.0, reduction="mean"):
        self.margin, self.reduction = margin, reduction

    def forward(self, x1, x2, y):
        return _reduce((-y * (x1.float() - x2.float()) + self.margin).clamp_min(0), self.reduction)


class TripletLoss(Loss):
    def __init__(self, margin=1.0, reduction="mean"):
        self.margin, self.reduction = margin, reduction

    def forward(self, a, p, n):
        dp = (a.float() - p.float()).norm(dim=-1)
        dn = (a.float() - n.float()).norm(dim=-1)
        return _reduce((dp - dn + self.margin).clamp_min(0), self.reduction)


class ContrastiveLoss(Loss):
    def __init__(self, margin=1.0, reduction="mean"):
        self.margin, self.reduction = margin, reduction

    def forward(self, x1, x2, same):
        d = (x1.float() - x2.float()).norm(dim=-1)
        s = same.float()
        return _reduce(s * d ** 2 + (1 - s) * (self.margin - d).clamp_min(0) ** 2, self.reduction)


class InfoNCELoss(Loss):
    """InfoNCE over a batch: positives on the diagonal of the query/key similarity matrix."""

    def __init__(self, temperature=0.07):
        self.t = temperature

    def forward(self, q, k):
        qn, kn = F.normalize(q.float(), dim=-1), F.normalize(k.float(), dim=-1)
        logits = qn @ kn.t() / self.t
        return F.cross_entropy(logits, torch.arange(q.shape[0], device=q.device))


class NTXentLoss(InfoNCELoss):
    """SimCLR NT-Xent: both views as anchors, all other 2N-2 samples as negatives."""

    def forward(self, z1, z2):
        z = F.normalize(torch.cat([z1, z2]).float(), dim=-1)
        n = z1.shape[0]
        sim = z @ z.t() / self.t
        sim.fill_diagonal_(float("-inf"))
        target = torch.cat([torch.arange(n, 2 * n), torch.arange(0, n)]).to(z.device)
        return F.cross_entropy(sim, target)


# ------------------------------------------------------------------ segmentation / adversarial / distillation
class DiceLoss(Loss):
    def __init__(self, smooth=1.0):
        self.smooth = smooth

    def forward(self, probs, target_onehot):
        p, t = probs.float().flatten(1), target_onehot.float().flatten(1)
        inter = (p * t).sum(1)
        return (1 - (2 * inter + self.smooth) / (p.sum(1) + t.sum(1) + self.smooth)).mean()


class CEDiceLoss(Loss):
    def __init__(self, ce_weight=0.5):
        self.w = ce_weight
        self.dice = DiceLoss()

    def forward(self, logits, target):
        ce = F.cross_entropy(logits.float(), target)
        probs = logits.float().softmax(1)
        oh = F.one_hot(target, logits.shape[1]).movedim(-1, 1)
        return self.w * ce + (1 - self.w) * self.dice(probs, oh)


class IoULoss(DiceLoss):
    def forward(self, probs, target):
        p, t = probs.float().flatten(1), target.float().flatten(1)
        inter = (p * t).sum(1)
        union = p.sum(1) + t.sum(1) - inter
        return (1 - (inter + self.smooth) / (union + self.smooth)).mean()


class WassersteinLoss(Loss):
    def forward(self, critic_real, critic_fake=None):
        return critic_fake.float().mean() - critic_real.float().mean() if critic_fake is not None \
            else -critic_real.float().mean()


class GANLoss(Loss):
    """Non-saturating GAN loss on discriminator logits (target True = real)."""

    def forward(self, logits, real: bool = True):
        t = torch.ones_like(logits) if real else torch.zeros_like(logits)
        return F.binary_cross_entropy_with_logits(logits.float(), t.float())


class HingeGANLoss(Loss):
    def forward(self, logits, real: bool = True):
        return F.relu(1 - logits.float()).mean() if real else F.relu(1 + logits.float()).mean()


class DistillationLoss(Loss):
    """alpha * T^2 KL(student_T || teacher_T) + (1 - alpha) * CE(student, labels)."""

    def __init__(self, temperature=2.0, alpha=0.5):
        self.T, self.alpha = temperature, alpha

    def forward(self, student, teacher, labels=None):
        T = self.T
        kd = F.kl_div(F.log_softmax(student.float() / T, -1), F.softmax(teacher.float() / T, -1),
                      reduction="batchmean") * T * T
        if labels is None:
            return kd
        return self.alpha * kd + (1 - self.alpha) * F.cross_entropy(student.float(), labels)


class MaskedLoss(Loss):
    """Apply any elementwise loss only where mask is set (masked.rs)."""

    def __init__(self, base: Loss):
        self.base = base
        base.reduction = "none"

    def forward(self, p, t, mask):
        v = self.base(p, t)
        m = mask.float()
        return (v * m).sum() / m.sum().clamp_min(1)


class CombinedLoss(Loss):
    """Weighted sum of losses (combine.rs)."""

    def __init__(self, *pairs):
        self.pairs = pairs

    def forward(self, p, t):
        return sum(w * l(p, t) for w, l in self.pairs)


LOSSES = {c.__name__: c for c in [CrossEntropyLoss, NLLLoss, BCELoss, BCEWithLogitsLoss, FocalLoss, HingeLoss,
                                 KLDivLoss, CTCLoss, MSELoss, L1Loss, HuberLoss, SmoothL1Loss, LogCoshLoss,
                                 QuantileLoss, PoissonNLLLoss, GaussianNLLLoss, CosineEmbeddingLoss,
                                 MarginRankingLoss, TripletLoss, ContrastiveLoss, InfoNCELoss, NTXentLoss, DiceLoss,
                                 CEDiceLoss, IoULoss, WassersteinLoss, GANLoss, HingeGANLoss, DistillationLoss]}


# ------------------------------------------------------------------ metric learning / robust / adversarial extras
class ArcFaceLoss(Loss):
    """Additive angular margin (Deng et al. 2019) on cosine logits [B, C]: the target class's logit is
    s cos(theta + m) with theta = acos(clamp(cos, -1, 1)), the others s cos; cross-entropy over the row
    (crates/brain-loss/src/metric_loss/mod.rs:30-74)."""

    def __init__(self, scale: float = 64.0, margin: float = 0.5, reduction: str = "mean"):
        self.s, self.m, self.reduction = scale, margin, reduction

    def forward(self, cos_thetas, targets):
        c = cos_thetas.clamp(-1.0, 1.0)
        t = targets.long()
        tgt = torch.cos(torch.acos(c.gather(1, t[:, None])) + self.m)
        logits = self.s * c.scatter(1, t[:, None], tgt)
        return _reduce(F.cross_entropy(logits, t, reduction="none"), self.reduction)


class AngularDistanceLoss(Loss):
    """acos of the cosine similarity between prediction and target rows, in radians."""

    def __init__(self, reduction: str = "mean"):
        self.reduction = reduction

    def forward(self, pred, target):
        cos = F.cosine_similarity(pred, target, dim=-1, eps=1e-12).clamp(-1.0, 1.0)
        return _reduce(torch.acos(cos), self.reduction)


class CauchyLoss(Loss):
    """0.5 c^2 ln(1 + r^2 / c^2) per residual r (robust to outliers; crates/brain-loss/src/regression/robust.rs)."""

    def __init__(self, c: float = 1.0, reduction: str = "mean"):
        self.c, self.reduction = c, reduction

    def forward(self, pred, target):
        if pred.shape != target.shape:
            raise ValueError(f"shape mismatch: {tuple(pred.shape)} vs {tuple(target.shape)}")
        c2 = self.c * self.c
        return _reduce(0.5 * c2 * torch.log1p((pred - target) ** 2 / c2), self.reduction)


class LSGANLoss:
    """Least-squares GAN: D: mean 0.5 (D(x) - 1)^2 + mean 0.5 D(G(z))^2; G: mean 0.5 (D(G(z)) - 1)^2."""

    @staticmethod
    def discriminator_loss(d_real, d_fake):
        return 0.5 * ((d_real - 1) ** 2).mean() + 0.5 * (d_fake ** 2).mean()

    @staticmethod
    def generator_loss(d_fake):
        return 0.5 * ((d_fake - 1) ** 2).mean()


class RelativisticLoss:
    """Relativistic average GAN losses with the logistic link: D pushes D(x) - mean D(G(z)) up and
    D(G(z)) - mean D(x) down; G the reverse."""

    @staticmethod
    def discriminator_loss(d_real, d_fake):
        return F.softplus(-(d_real - d_fake.mean())).mean() + F.softplus(d_fake - d_real.mean()).mean()

    @staticmethod
    def generator_loss(d_real, d_fake):
        return F.softplus(-(d_fake - d_real.mean())).mean() + F.softplus(d_real - d_fake.mean()).mean()


# ------------------------------------------------------------------ the reference's spellings and helpers
# crates/brain-loss/src: regression/mse.rs (MAELoss), classification/other.rs (KLDivergenceLoss),
# distillation.rs (KnowledgeDistillationLoss), contrastive/simclr.rs (SimCLRLoss), contrastive/triplet.rs
# (TripletMarginLoss), adversarial/{mod,other}.rs, combine.rs (CompositeLoss), masked.rs (apply_loss_mask),
# ops.rs (one_hot_target, log_sum_exp_2d), utils.rs (reduction_apply, weighted_average, clamp_eps).
MAELoss = L1Loss
KLDivergenceLoss = KLDivLoss
KnowledgeDistillationLoss = DistillationLoss
SimCLRLoss = NTXentLoss
TripletMarginLoss = TripletLoss
AdversarialLoss = GANLoss
HingeAdversarialLoss = HingeGANLoss
CompositeLoss = CombinedLoss


def apply_loss_mask(per_element: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """Mean of the per-element loss over the positions where mask is nonzero (0 when none are)."""
    m = mask.to(per_element.dtype)
    return (per_element * m).sum() / m.sum().clamp_min(1.0)


def one_hot_target(indices: torch.Tensor, num_classes: int, dtype=torch.float32) -> torch.Tensor:
    return torch.nn.functional.one_hot(indices.long(), num_classes).to(dtype)


def log_sum_exp_2d(x: torch.Tensor) -> torch.Tensor:
    """Row-wise log-sum-exp of a [N, C] matrix (max-shifted)."""
    return torch.logsumexp(x, dim=-1)


def reduction_apply(x: torch.Tensor, reduction: str = "mean") -> torch.Tensor:
    return _reduce(x, reduction)


def weighted_average(values: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    w = weights.to(values.dtype)
    return (values * w).sum() / w.sum().clamp_min(torch.finfo(values.dtype).tiny)


def clamp_eps(x: torch.Tensor, eps: float = 1e-7) -> torch.Tensor:
    return x.clamp(eps, 1 - eps)


_LOSSES = {"mse": MSELoss, "mae": L1Loss, "l1": L1Loss, "huber": HuberLoss, "smooth_l1": SmoothL1Loss,
           "log_cosh": LogCoshLoss, "cross_entropy": CrossEntropyLoss, "nll": NLLLoss, "bce": BCELoss,
           "bce_with_logits": BCEWithLogitsLoss, "focal": FocalLoss, "hinge": HingeLoss, "kl_div": KLDivLoss,
           "dice": DiceLoss, "iou": IoULoss, "cosine_embedding": CosineEmbeddingLoss}


def loss_names() -> list[str]:
    return sorted(_LOSSES)


def compute_loss(kind: str, pred: torch.Tensor, target: torch.Tensor, **kw) -> torch.Tensor:
    """One call by name: ``compute_loss("huber", pred, target, delta=0.5)``."""
    if kind not in _LOSSES:
        raise ValueError(f"unknown loss {kind!r}; known: {', '.join(loss_names())}")
    return _LOSSES[kind](**kw)(pred, target)
