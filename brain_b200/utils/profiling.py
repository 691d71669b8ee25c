"""Profiling utilities (reference brain-utils prof: Profiler.record_span, TimingStats mean/p50/p95/p99,
TimingTree, AtomicCounter/Gauge, ScopeGuard; crates/brain-utils/src/prof/*.rs and brain-benchmark).

GPU timing uses CUDA events on the current stream (``CudaTimer``), with an optional NVTX range so
spans show up in external profilers; ``max_over_ranks`` reduces a per-rank time to the slowest rank.
"""
from __future__ import annotations

import contextlib
import statistics
import threading
import time

import torch


class TimingStats:
    def __init__(self):
        self.samples: list[float] = []

    def add(self, v: float) -> None:
        self.samples.append(float(v))

    def _pct(self, q: float) -> float:
        s = sorted(self.samples)
        if not s:
            return float("nan")
        k = (len(s) - 1) * q
        lo, hi = int(k), min(int(k) + 1, len(s) - 1)
        return s[lo] + (s[hi] - s[lo]) * (k - lo)

    def summary(self) -> dict:
        if not self.samples:
            return {"count": 0}
        return {"count": len(self.samples), "mean": statistics.fmean(self.samples), "min": min(self.samples),
                "max": max(self.samples), "p50": self._pct(0.5), "p95": self._pct(0.95), "p99": self._pct(0.99)}


class Profiler:
    """Named spans (wall clock on the host, or CUDA events when ``cuda=True``)."""

    def __init__(self, cuda: bool = False, nvtx: bool = False):
        self.cuda = cuda and torch.cuda.is_available()
        self.nvtx = nvtx and torch.cuda.is_available()
        self.stats: dict[str, TimingStats] = {}
        self._pending: list = []

    @contextlib.contextmanager
    def span(self, name: str):
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        if self.cuda:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            try:
                yield
            finally:
                e.record()
                self._pending.append((name, s, e))
        else:
            t0 = time.perf_counter()
            try:
                yield
            finally:
                self.stats.setdefault(name, TimingStats()).add((time.perf_counter() - t0) * 1e3)
        if self.nvtx:
            torch.cuda.nvtx.range_pop()

    record_span = span

    def flush(self) -> None:
        if self._pending:
            torch.cuda.synchronize()
            for name, s, e in self._pending:
                self.stats.setdefault(name, TimingStats()).add(s.elapsed_time(e))
            self._pending.clear()

    def report(self) -> dict:
        self.flush()
        return {k: v.summary() for k, v in self.stats.items()}


class CudaTimer:
    """Device time of a region in ms (events on the current stream, synchronised on exit)."""

    def __enter__(self):
        torch.cuda.synchronize()
        self.s, self.e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.s.record()
        return self

    def __exit__(self, *a):
        self.e.record()
        torch.cuda.synchronize()
        self.ms = self.s.elapsed_time(self.e)


def max_over_ranks(value: float, device=None) -> float:
    import torch.distributed as dist
    if not dist.is_initialized():
        return value
    t = torch.tensor([value], device=device or ("cuda" if torch.cuda.is_available() else "cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class AtomicCounter:
    def __init__(self, v: int = 0):
        self._v, self._lock = v, threading.Lock()

    def add(self, d: int = 1) -> int:
        with self._lock:
            self._v += d
            return self._v

    def get(self) -> int:
        return self._v


class Gauge(AtomicCounter):
    def set(self, v) -> None:
        with self._lock:
            self._v = v


class ScopeGuard:
    def __init__(self, fn):
        self.fn = fn

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.fn()
