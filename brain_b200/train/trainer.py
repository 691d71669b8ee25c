"""Trainer with the reference's API (crates/brain-train/src/lib.rs:116-1400).

``TrainerBuilder().model(m).loss(...).optimizer(...).learning_rate(lr).regularizer(r).build()`` ->
``Trainer`` with ``train_batch(batch) -> TrainStep{loss, accuracy, optimizer: StepInfo}``,
``fit(batches, epochs)``, ``fit_accumulated(batches, epochs, accumulation)``, ``evaluate``,
``summary``, ``state()`` / ``load_state()`` (``ModelState`` / ``.brain``). ``Batch{inputs, targets}``
and ``SyntheticClassification.two_class_points`` mirror lib.rs:116-200. The model is any module
(the reference's own Sequential of Linear/ReLU/Conv2d/Pool/Flatten maps to ``nn.Sequential``), the
backward pass is autograd over the sm_100a ops, and the default optimizer is SGD with lr 0.1 as in
the reference. Regularizers contribute extra gradients (L2 ``weight * p``) like lib.rs:1247-1258.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import torch

from ..checkpoint.formats import ModelState
from ..ops import cross_entropy
from ..optim.optimizers import SGD, Optimizer, StepInfo
from .callbacks import TrainingCallback


@dataclass
class Batch:
    inputs: torch.Tensor
    targets: torch.Tensor

    def __post_init__(self):
        if self.inputs.dim() == 0 or self.inputs.shape[0] != len(self.targets):
            raise ValueError(f"batch shape mismatch: inputs {tuple(self.inputs.shape)}, targets {len(self.targets)}")
        if not isinstance(self.targets, torch.Tensor):
            self.targets = torch.as_tensor(self.targets, dtype=torch.long)

    def target_tensor(self) -> torch.Tensor:
        return self.targets.double()

    def to(self, device):
        return Batch(self.inputs.to(device), self.targets.to(device))


class SyntheticClassification:
    """Deterministic 2-class points: class 0 around (-1,-1), class 1 around (+1,+1)."""

    def __init__(self, inputs: torch.Tensor, targets: torch.Tensor):
        self.inputs, self.targets = inputs, targets

    @staticmethod
    def two_class_points(n: int = 64, seed: int = 0) -> "SyntheticClassification":
        g = torch.Generator().manual_seed(seed)
        y = torch.arange(n) % 2
        centre = (y.float() * 2 - 1)[:, None].expand(n, 2)
        x = centre + 0.3 * torch.randn(n, 2, generator=g)
        return SyntheticClassification(x, y)

    def batches(self, batch_size: int) -> list[Batch]:
        return [Batch(self.inputs[i:i + batch_size], self.targets[i:i + batch_size])
                for i in range(0, len(self.targets), batch_size)]


@dataclass
class TrainStep:
    loss: float
    accuracy: float
    optimizer: StepInfo


@dataclass
class TrainingSummary:
    steps: int = 0
    loss: float = 0.0
    accuracy: float = 0.0
    history: list = field(default_factory=list)
    seconds: float = 0.0


class L2Regularizer:
    def __init__(self, weight: float):
        self.weight = weight

    def gradients(self, params):
        return [self.weight * p.detach() for p in params]

    def penalty(self, params) -> float:
        return 0.5 * self.weight * sum(float(p.detach().float().pow(2).sum()) for p in params)


class L1Regularizer(L2Regularizer):
    def gradients(self, params):
        return [self.weight * p.detach().sign() for p in params]

    def penalty(self, params) -> float:
        return self.weight * sum(float(p.detach().abs().sum()) for p in params)


class Trainer:
    def __init__(self, model: torch.nn.Module, loss=None, optimizer: Optimizer | None = None, regularizers=None,
                 callbacks: list[TrainingCallback] | None = None, device=None):
        self.model = model
        self.loss_fn = loss or (lambda logits, t: cross_entropy(logits, t))
        self.optimizer = optimizer or SGD(model.parameters(), lr=0.1)
        self.regularizers = list(regularizers or [])
        self.callbacks = list(callbacks or [])
        self.device = device
        self.steps = 0
        self._hist: list[TrainStep] = []

    @staticmethod
    def builder() -> "TrainerBuilder":
        return TrainerBuilder()

    def _move(self, batch: Batch) -> Batch:
        return batch.to(self.device) if self.device is not None else batch

    def _forward_loss(self, batch: Batch):
        logits = self.model(batch.inputs)
        loss = self.loss_fn(logits, batch.targets)
        return logits, loss

    def _apply_regularizers(self):
        if not self.regularizers:
            return
        params = [p for p in self.model.parameters() if p.requires_grad]
        for r in self.regularizers:
            for p, g in zip(params, r.gradients(params)):
                if p.grad is None:
                    p.grad = g.to(p.dtype).clone()
                else:
                    p.grad.add_(g.to(p.grad.dtype))

    @staticmethod
    def _accuracy(logits, targets) -> float:
        if logits.dim() < 2:
            return float("nan")
        pred = logits.detach().argmax(-1)
        return float((pred == targets).float().mean())

    def train_batch(self, batch: Batch) -> TrainStep:
        self.model.train()
        batch = self._move(batch)
        self.optimizer.zero_grad()
        logits, loss = self._forward_loss(batch)
        loss.backward()
        self._apply_regularizers()
        info = self.optimizer.step()
        self.steps += 1
        st = TrainStep(float(loss.detach()), self._accuracy(logits, batch.targets), info)
        self._hist.append(st)
        for cb in self.callbacks:
            cb.on_step_end(self, st)
        return st

    def fit(self, batches: list[Batch], epochs: int = 1) -> TrainingSummary:
        return self.fit_accumulated(batches, epochs, 1)

    def fit_accumulated(self, batches: list[Batch], epochs: int = 1, accumulation: int = 1) -> TrainingSummary:
        t0 = time.time()
        out = TrainingSummary()
        for ep in range(epochs):
            for cb in self.callbacks:
                cb.on_epoch_start(self, ep)
            ep_losses = []
            if accumulation <= 1:
                for b in batches:
                    st = self.train_batch(b)
                    ep_losses.append(st.loss)
                    out.history.append(st)
            else:
                self.model.train()
                for i in range(0, len(batches), accumulation):
                    group = [self._move(b) for b in batches[i:i + accumulation]]
                    self.optimizer.zero_grad()
                    tot, acc = 0.0, 0.0
                    for b in group:
                        logits, loss = self._forward_loss(b)
                        (loss / len(group)).backward()
                        tot += float(loss.detach()) / len(group)
                        acc += self._accuracy(logits, b.targets) / len(group)
                    self._apply_regularizers()
                    info = self.optimizer.step()
                    self.steps += 1
                    st = TrainStep(tot, acc, info)
                    out.history.append(st)
                    ep_losses.append(tot)
            stop = False
            for cb in self.callbacks:
                stop |= bool(cb.on_epoch_end(self, ep, sum(ep_losses) / max(1, len(ep_losses))))
            if stop:
                break
        out.steps = len(out.history)
        if out.history:
            out.loss = sum(s.loss for s in out.history) / out.steps
            out.accuracy = sum(s.accuracy for s in out.history) / out.steps
        out.seconds = time.time() - t0
        return out

    @torch.no_grad()
    def evaluate(self, batches: list[Batch]) -> tuple[float, float]:
        self.model.eval()
        tl, ta, n = 0.0, 0.0, 0
        for b in batches:
            b = self._move(b)
            logits, loss = self._forward_loss(b)
            k = len(b.targets)
            tl += float(loss) * k
            ta += self._accuracy(logits, b.targets) * k
            n += k
        return tl / max(1, n), ta / max(1, n)

    def summary(self) -> TrainingSummary:
        h = self._hist
        if not h:
            return TrainingSummary()
        return TrainingSummary(len(h), sum(s.loss for s in h) / len(h), sum(s.accuracy for s in h) / len(h), list(h))

    def state(self, metadata: dict | None = None) -> ModelState:
        md = {"format": "brain-train-state-v1", "optimizer_steps": str(self.steps),
              "layers": str(sum(1 for _ in self.model.modules()) - 1)}
        md.update(metadata or {})
        return ModelState.from_module(self.model, md)

    def load_state(self, state: ModelState) -> None:
        state.load_into(self.model)
        self.steps = int(state.metadata.get("optimizer_steps", self.steps))


class TrainerBuilder:
    def __init__(self):
        self._model = None
        self._loss = None
        self._opt = None
        self._opt_factory = None
        self._lr = 0.1
        self._regs = []
        self._callbacks = []
        self._device = None

    def model(self, m):
        self._model = m
        return self

    def loss(self, fn):
        self._loss = fn
        return self

    def optimizer(self, opt_or_factory):
        if isinstance(opt_or_factory, Optimizer):
            self._opt = opt_or_factory
        else:
            self._opt_factory = opt_or_factory
        return self

    def learning_rate(self, lr: float):
        self._lr = lr
        return self

    def regularizer(self, r):
        self._regs.append(r)
        return self

    def callback(self, cb):
        self._callbacks.append(cb)
        return self

    def device(self, d):
        self._device = d
        return self

    def build(self) -> Trainer:
        if self._model is None:
            raise ValueError("TrainerBuilder: model is required")
        opt = self._opt
        if opt is None:
            factory = self._opt_factory or SGD
            opt = factory(self._model.parameters(), lr=self._lr)
        return Trainer(self._model, self._loss, opt, self._regs, self._callbacks, self._device)


def perplexity(loss: float) -> float:
    return math.exp(min(loss, 50.0))
