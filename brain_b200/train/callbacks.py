"""Training callbacks, metrics and checkpoint tracking (crates/brain-train/src/callbacks.rs:19-131,
metrics.rs, checkpointer.rs:9-62): ``EarlyStopping``, ``MetricHistoryLogger``, ``AccuracyMetric``,
``RunningAverage``, ``TopKAccuracyMetric``, ``BestModelTracker``, ``CheckpointMeta``, plus a JSONL
step logger with the rank prefix used by the distributed runs."""
from __future__ import annotations

import json
import math
from dataclasses import dataclass

import torch


class TrainingCallback:
    def on_epoch_start(self, trainer, epoch: int) -> None:
        pass

    def on_step_end(self, trainer, step) -> None:
        pass

    def on_epoch_end(self, trainer, epoch: int, loss: float) -> bool:
        """Return True to stop training."""
        return False


class EarlyStopping(TrainingCallback):
    def __init__(self, patience: int = 3, min_delta: float = 0.0):
        self.patience, self.min_delta = patience, min_delta
        self.best = math.inf
        self.bad = 0
        self.stopped_epoch = None

    def on_epoch_end(self, trainer, epoch, loss):
        if loss < self.best - self.min_delta:
            self.best, self.bad = loss, 0
            return False
        self.bad += 1
        if self.bad >= self.patience:
            self.stopped_epoch = epoch
            return True
        return False


class MetricHistoryLogger(TrainingCallback):
    def __init__(self):
        self.losses: list[float] = []
        self.accuracies: list[float] = []
        self.epoch_losses: list[float] = []

    def on_step_end(self, trainer, step):
        self.losses.append(step.loss)
        self.accuracies.append(step.accuracy)

    def on_epoch_end(self, trainer, epoch, loss):
        self.epoch_losses.append(loss)
        return False


class JsonlStepLogger(TrainingCallback):
    def __init__(self, path: str, rank: int = 0):
        self.f = open(path, "a")
        self.rank = rank

    def on_step_end(self, trainer, step):
        self.f.write(json.dumps({"rank": self.rank, "step": trainer.steps, "loss": step.loss, "acc": step.accuracy,
                                 "grad_norm": step.optimizer.grad_norm, "lr": step.optimizer.lr}) + "\n")
        self.f.flush()


class RunningAverage:
    def __init__(self):
        self.total, self.count = 0.0, 0

    def update(self, v: float, n: int = 1):
        self.total += v * n
        self.count += n

    def value(self) -> float:
        return self.total / self.count if self.count else 0.0

    def reset(self):
        self.total, self.count = 0.0, 0


class AccuracyMetric(RunningAverage):
    def update_logits(self, logits: torch.Tensor, targets: torch.Tensor):
        pred = logits.argmax(-1)
        self.total += float((pred == targets).sum())
        self.count += targets.numel()


class TopKAccuracyMetric(RunningAverage):
    def __init__(self, k: int = 5):
        super().__init__()
        self.k = k

    def update_logits(self, logits, targets):
        top = logits.topk(self.k, -1).indices
        self.total += float((top == targets[..., None]).any(-1).sum())
        self.count += targets.numel()


@dataclass
class CheckpointMeta:
    epoch: int
    step: int
    metric: float
    path: str


class BestModelTracker:
    def __init__(self, mode: str = "min"):
        self.mode = mode
        self.best: CheckpointMeta | None = None

    def update(self, meta: CheckpointMeta) -> bool:
        better = self.best is None or (meta.metric < self.best.metric if self.mode == "min"
                                       else meta.metric > self.best.metric)
        if better:
            self.best = meta
        return better


class PeriodicCheckpointer(TrainingCallback):
    """Saves ``trainer.state()`` as a ``.brain`` text checkpoint every ``every`` epochs (and the best
    epoch by loss as ``best.brain``), keeping the ``keep_last`` most recent periodic files
    (reference checkpointer.rs:9-62 with ``BestModelTracker``). ``latest()`` returns the newest path
    for resuming with ``Trainer.load_state(ModelState.load_file(path))``."""

    def __init__(self, directory: str, every: int = 1, keep_last: int = 3):
        import os

        os.makedirs(directory, exist_ok=True)
        self.dir, self.every, self.keep_last = directory, max(1, every), keep_last
        self.saved: list[str] = []
        self.best = BestModelTracker("min")

    def on_epoch_end(self, trainer, epoch, loss):
        import os

        if (epoch + 1) % self.every == 0:
            path = os.path.join(self.dir, f"epoch{epoch + 1:06d}.brain")
            trainer.state({"epoch": str(epoch + 1), "loss": repr(float(loss))}).save_file(path)
            self.saved.append(path)
            while len(self.saved) > self.keep_last:
                old = self.saved.pop(0)
                if os.path.exists(old):
                    os.remove(old)
        if self.best.update(CheckpointMeta(epoch + 1, 0, float(loss), os.path.join(self.dir, "best.brain"))):
            trainer.state({"epoch": str(epoch + 1), "loss": repr(float(loss))}).save_file(self.best.best.path)
        return False

    def latest(self):
        return self.saved[-1] if self.saved else None


# ------------------------------------------------------------------ the reference's remaining names
# crates/brain-train/src: callbacks.rs (CallbackAction), checkpointer.rs (check_improvement), lib.rs
# (argmax_rows, L2Regularization, TrainableModule / TensorModuleAdapter), metrics.rs (windowed averages).

class CallbackAction:
    """What a callback asks of the loop: keep going or stop."""
    CONTINUE, STOP = "continue", "stop"

    @staticmethod
    def from_bool(stop: bool) -> str:
        return CallbackAction.STOP if stop else CallbackAction.CONTINUE


def check_improvement(new: float, best: float | None, mode: str = "min", min_delta: float = 0.0) -> bool:
    if best is None:
        return True
    return new < best - min_delta if mode == "min" else new > best + min_delta


def argmax_rows(x) -> list[int]:
    import torch
    return torch.as_tensor(x).argmax(-1).tolist()


class WindowedAverage:
    """Mean of the last ``window`` values (the reference's RunningAverage with_window)."""

    def __init__(self, window: int = 100):
        from collections import deque
        self.window, self.values = window, deque(maxlen=window)

    def update(self, v: float) -> float:
        self.values.append(float(v))
        return self.value

    @property
    def value(self) -> float:
        return sum(self.values) / len(self.values) if self.values else 0.0


class TensorModuleAdapter:
    """Wraps a plain function of tensors as a trainable module: parameters are the given tensors."""

    def __init__(self, fn, params):
        self.fn, self._params = fn, list(params)

    def parameters(self):
        return iter(self._params)

    def __call__(self, *args):
        return self.fn(*args)


TrainableModule = TensorModuleAdapter
