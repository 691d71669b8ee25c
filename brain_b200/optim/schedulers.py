"""Learning-rate schedulers (crates/brain-optim/src/schedulers/*.rs).

Each scheduler exposes ``lr_at(step)`` (pure) and ``step()`` which advances and writes the new rate
into the optimizer through ``set_lr`` (works for every optimizer here, including ``FlatAdamW``).
Covered: constant, step, multi-step, exponential, polynomial, cosine annealing, cosine with warm
restarts, cyclic (triangular / triangular2 / exp_range), one-cycle, reduce-on-plateau, and linear /
constant / exponential warmup wrappers.
"""
from __future__ import annotations

import math


class LRScheduler:
    def __init__(self, optimizer, base_lr: float | None = None):
        self.optimizer = optimizer
        self.base_lr = base_lr if base_lr is not None else optimizer.get_lr()
        self.last_step = 0

    def lr_at(self, step: int) -> float:  # pragma: no cover - abstract
        raise NotImplementedError

    def get_lr(self) -> float:
        return self.lr_at(self.last_step)

    def step(self, *_):
        self.last_step += 1
        lr = self.lr_at(self.last_step)
        self.optimizer.set_lr(lr)
        return lr

    def state_dict(self):
        return {"last_step": self.last_step, "base_lr": self.base_lr}

    def load_state_dict(self, sd):
        self.last_step, self.base_lr = sd["last_step"], sd["base_lr"]


class ConstantLR(LRScheduler):
    def lr_at(self, step):
        return self.base_lr


class StepLR(LRScheduler):
    def __init__(self, optimizer, step_size: int, gamma: float = 0.1):
        super().__init__(optimizer)
        self.step_size, self.gamma = step_size, gamma

    def lr_at(self, step):
        return self.base_lr * self.gamma ** (step // self.step_size)


class MultiStepLR(LRScheduler):
    def __init__(self, optimizer, milestones, gamma: float = 0.1):
        super().__init__(optimizer)
        self.milestones, self.gamma = sorted(milestones), gamma

    def lr_at(self, step):
        return self.base_lr * self.gamma ** sum(1 for m in self.milestones if step >= m)


class ExponentialLR(LRScheduler):
    def __init__(self, optimizer, gamma: float):
        super().__init__(optimizer)
        self.gamma = gamma

    def lr_at(self, step):
        return self.base_lr * self.gamma ** step


class PolynomialLR(LRScheduler):
    def __init__(self, optimizer, total_steps: int, power: float = 1.0, end_lr: float = 0.0):
        super().__init__(optimizer)
        self.total, self.power, self.end_lr = total_steps, power, end_lr

    def lr_at(self, step):
        t = min(step, self.total) / max(1, self.total)
        return (self.base_lr - self.end_lr) * (1 - t) ** self.power + self.end_lr


class CosineAnnealingLR(LRScheduler):
    def __init__(self, optimizer, t_max: int, eta_min: float = 0.0):
        super().__init__(optimizer)
        self.t_max, self.eta_min = t_max, eta_min

    def lr_at(self, step):
        t = min(step, self.t_max)
        return self.eta_min + (self.base_lr - self.eta_min) * (1 + math.cos(math.pi * t / self.t_max)) / 2


class CosineAnnealingWarmRestarts(LRScheduler):
    def __init__(self, optimizer, t_0: int, t_mult: int = 1, eta_min: float = 0.0):
        super().__init__(optimizer)
        self.t_0, self.t_mult, self.eta_min = t_0, t_mult, eta_min

    def lr_at(self, step):
        t, period = step, self.t_0
        while t >= period:
            t -= period
            period *= self.t_mult
        return self.eta_min + (self.base_lr - self.eta_min) * (1 + math.cos(math.pi * t / period)) / 2


class CyclicLR(LRScheduler):
    def __init__(self, optimizer, base_lr: float, max_lr: float, step_size_up: int = 2000, mode: str = "triangular",
                 gamma: float = 1.0):
        super().__init__(optimizer, base_lr)
        self.max_lr, self.up, self.mode, self.gamma = max_lr, step_size_up, mode, gamma

    def lr_at(self, step):
        cycle = math.floor(1 + step / (2 * self.up))
        x = abs(step / self.up - 2 * cycle + 1)
        amp = (self.max_lr - self.base_lr) * max(0.0, 1 - x)
        if self.mode == "triangular2":
            amp /= 2 ** (cycle - 1)
        elif self.mode == "exp_range":
            amp *= self.gamma ** step
        return self.base_lr + amp


class OneCycleLR(LRScheduler):
    def __init__(self, optimizer, max_lr: float, total_steps: int, pct_start: float = 0.3, div_factor: float = 25.0,
                 final_div_factor: float = 1e4):
        super().__init__(optimizer, max_lr / div_factor)
        self.max_lr, self.total, self.pct = max_lr, total_steps, pct_start
        self.final = self.base_lr / final_div_factor

    def lr_at(self, step):
        up = max(1, int(self.pct * self.total))
        if step <= up:
            return self.base_lr + (self.max_lr - self.base_lr) * (1 - math.cos(math.pi * step / up)) / 2
        t = min(1.0, (step - up) / max(1, self.total - up))
        return self.final + (self.max_lr - self.final) * (1 + math.cos(math.pi * t)) / 2


class ReduceLROnPlateau(LRScheduler):
    def __init__(self, optimizer, mode: str = "min", factor: float = 0.1, patience: int = 10, threshold: float = 1e-4,
                 min_lr: float = 0.0):
        super().__init__(optimizer)
        self.mode, self.factor, self.patience, self.threshold, self.min_lr = mode, factor, patience, threshold, min_lr
        self.best = math.inf if mode == "min" else -math.inf
        self.bad = 0
        self.lr = self.base_lr

    def lr_at(self, step):
        return self.lr

    def step(self, metric: float = None):
        self.last_step += 1
        if metric is None:
            return self.lr
        better = metric < self.best * (1 - self.threshold) if self.mode == "min" else \
            metric > self.best * (1 + self.threshold)
        if better:
            self.best, self.bad = metric, 0
        else:
            self.bad += 1
            if self.bad > self.patience:
                self.lr = max(self.min_lr, self.lr * self.factor)
                self.bad = 0
        self.optimizer.set_lr(self.lr)
        return self.lr


class WarmupScheduler(LRScheduler):
    """Warmup for ``warmup_steps`` (linear / constant / exponential), then the wrapped schedule."""

    def __init__(self, optimizer, warmup_steps: int, after: LRScheduler | None = None, kind: str = "linear",
                 start_factor: float = 0.0):
        super().__init__(optimizer)
        self.warmup, self.after, self.kind, self.start = warmup_steps, after, kind, start_factor

    def lr_at(self, step):
        if step < self.warmup:
            f = step / max(1, self.warmup)
            if self.kind == "linear":
                return self.base_lr * (self.start + (1 - self.start) * f)
            if self.kind == "constant":
                return self.base_lr * max(self.start, 1e-12)
            return self.base_lr * (max(self.start, 1e-3) ** (1 - f))
        if self.after is None:
            return self.base_lr
        return self.after.lr_at(step - self.warmup)


def LinearWarmup(optimizer, warmup_steps, after=None):
    return WarmupScheduler(optimizer, warmup_steps, after, "linear")


def ConstantWarmup(optimizer, warmup_steps, after=None, factor=0.1):
    return WarmupScheduler(optimizer, warmup_steps, after, "constant", factor)


def ExponentialWarmup(optimizer, warmup_steps, after=None):
    return WarmupScheduler(optimizer, warmup_steps, after, "exponential")


def warmup_cosine(optimizer, warmup_steps: int, total_steps: int, eta_min: float = 0.0):
    return WarmupScheduler(optimizer, warmup_steps,
                           CosineAnnealingLR(optimizer, max(1, total_steps - warmup_steps), eta_min))


class LRFinder:
    """Exponentially increasing learning rate range test: returns (lrs, losses)."""

    def __init__(self, optimizer, start_lr=1e-7, end_lr=10.0, num_steps=100):
        self.opt, self.start, self.end, self.n = optimizer, start_lr, end_lr, num_steps

    def run(self, step_fn):
        lrs, losses = [], []
        for i in range(self.n):
            lr = self.start * (self.end / self.start) ** (i / max(1, self.n - 1))
            self.opt.set_lr(lr)
            loss = float(step_fn())
            lrs.append(lr)
            losses.append(loss)
            if not math.isfinite(loss) or (losses and loss > 4 * min(losses)):
                break
        return lrs, losses


class NoamLR(LRScheduler):
    """Transformer schedule (Vaswani et al. 2017): factor d_model^-0.5 min(s^-0.5, s warmup^-1.5) with
    s = max(step, 1) (crates/brain-optim/src/schedulers/warmup.rs, NoamLR)."""

    def __init__(self, optimizer, d_model: int, warmup_steps: int = 4000, factor: float = 1.0):
        super().__init__(optimizer)
        self.d, self.w, self.f = d_model, max(warmup_steps, 1), factor

    def lr_at(self, step: int) -> float:
        s = max(step, 1)
        return self.f * self.d ** -0.5 * min(s ** -0.5, s * self.w ** -1.5)


class ChainedScheduler:
    """Several schedulers stepped together; each one's lr_at acts as a multiplicative factor on the base
    learning rate relative to its own base, so e.g. warmup x cosine compose."""

    def __init__(self, optimizer, schedulers):
        self.optimizer, self.schedulers = optimizer, list(schedulers)
        self.base_lr = optimizer.get_lr()
        self.last_step = 0

    def lr_at(self, step: int) -> float:
        lr = self.base_lr
        for s in self.schedulers:
            lr *= s.lr_at(step) / s.base_lr if s.base_lr else 1.0
        return lr

    def get_lr(self) -> float:
        return self.lr_at(self.last_step)

    def step(self, *_):
        self.last_step += 1
        for s in self.schedulers:
            s.last_step = self.last_step
        lr = self.lr_at(self.last_step)
        self.optimizer.set_lr(lr)
        return lr
