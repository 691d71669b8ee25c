"""Failure detection and fault policies (reference: ``FaultPolicy::{Retry, FailFast, ExcludeRank}`` enum
only, crates/brain-distributed/src/fault.rs:7-12; ``DistributedConfig.timeout_ms = 30000`` unused,
config.rs:19-28).

* ``Heartbeat``: every rank bumps a counter in the process-group store from a background thread;
  ``dead_ranks`` reports ranks whose counter stopped advancing for longer than the timeout.
* ``run_step_with_policy``: executes one training step and applies the policy when it raises
  (a collective timeout surfaces as an exception because every group has a bounded timeout, and the
  in-kernel NVLink waits report ``PeerTimeout``):
    FailFast     re-raise immediately;
    Retry        restore the last in-memory snapshot of the model/optimizer state and re-run, up to N times;
    ExcludeRank  report the dead ranks so the caller can rebuild the data-parallel group without them.
All failure injection in the tests happens on the host (a rank that raises, exits or never joins).
"""
from __future__ import annotations

import copy
import enum
import threading
import time

import torch


class FaultPolicy(enum.Enum):
    RETRY = "retry"
    FAIL_FAST = "fail_fast"
    EXCLUDE_RANK = "exclude_rank"


class StepFailed(RuntimeError):
    def __init__(self, msg, dead_ranks=None):
        super().__init__(msg)
        self.dead_ranks = dead_ranks or []


class Heartbeat:
    def __init__(self, store, rank: int, world: int, interval_s: float = 0.5, timeout_s: float = 5.0,
                 prefix: str = "brain_hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout, self.prefix = interval_s, timeout_s, prefix
        self._stop = threading.Event()
        self._seen: dict[int, tuple[int, float]] = {}
        self._thread = threading.Thread(target=self._run, daemon=True)

    def start(self):
        self._thread.start()
        return self

    def _run(self):
        n = 0
        while not self._stop.is_set():
            n += 1
            try:
                self.store.set(f"{self.prefix}/{self.rank}", str(n))
            except Exception:
                return
            self._stop.wait(self.interval)

    def stop(self):
        self._stop.set()

    def dead_ranks(self) -> list[int]:
        now = time.time()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                v = int(self.store.get(f"{self.prefix}/{r}")) if self._has(r) else 0
            except Exception:
                v = 0
            last_v, last_t = self._seen.get(r, (-1, now))
            if v != last_v:
                self._seen[r] = (v, now)
            elif now - last_t > self.timeout:
                dead.append(r)
        return dead

    def _has(self, r) -> bool:
        try:
            return bool(self.store.check([f"{self.prefix}/{r}"]))
        except Exception:
            return False


def snapshot(model: torch.nn.Module, optimizer=None) -> dict:
    return {"model": copy.deepcopy({k: v.detach().clone() for k, v in model.state_dict().items()}),
            "opt": copy.deepcopy(optimizer.state_dict()) if optimizer is not None else None}


def restore(snap: dict, model: torch.nn.Module, optimizer=None) -> None:
    model.load_state_dict(snap["model"])
    if optimizer is not None and snap["opt"] is not None:
        optimizer.load_state_dict(snap["opt"])


def run_step_with_policy(step_fn, policy: FaultPolicy, model=None, optimizer=None, retries: int = 2,
                         heartbeat: Heartbeat | None = None):
    snap = snapshot(model, optimizer) if (policy == FaultPolicy.RETRY and model is not None) else None
    attempt = 0
    while True:
        try:
            return step_fn()
        except Exception as e:  # noqa: BLE001 - every failure goes through the policy
            if policy == FaultPolicy.FAIL_FAST:
                raise
            if policy == FaultPolicy.EXCLUDE_RANK:
                dead = heartbeat.dead_ranks() if heartbeat is not None else []
                raise StepFailed(f"step failed ({e}); excluding ranks {dead}", dead) from e
            attempt += 1
            if attempt > retries:
                raise StepFailed(f"step failed after {retries} retries: {e}") from e
            if snap is not None:
                restore(snap, model, optimizer)
