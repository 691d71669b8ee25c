"""Benchmark harness: runner (warm-up, batch discovery, sweeps), statistics, A/B comparison with
Welch's t-test, a regression baseline store, hardware probe, energy estimate, log-bucket histogram,
reports (console / Markdown / CSV / JSON / HTML) and Prometheus / OpenTelemetry exporters, and a
kernel suite that times the framework's own kernels.

Reference: crates/brain-benchmark (runner.rs:13-110, statistics.rs:9-180, compare.rs:10-100,
baseline.rs:13-60, hardware.rs:11-90, energy.rs:8-20, histogram.rs:7-80, report.rs:10-140,
export.rs:8-60, kernels.rs:14-64).

Differences by design: GPU work is timed with CUDA events on the launching stream (synchronised on
both sides), never by host clock alone; the Welch test uses the Welch–Satterthwaite degrees of freedom
and the Student-t tail (scipy) rather than a normal approximation; energy comes from sampled NVML board
power when NVML is readable (read-only queries), else from a stated wattage.
"""
from __future__ import annotations

import json
import math
import os
import platform
import time
from dataclasses import asdict, dataclass, field

import torch


@dataclass
class BenchConfig:
    name: str
    warmup_iters: int = 3
    measure_iters: int = 20
    batch_size: int = 1
    device: str | None = None  # "cuda" -> CUDA-event timing
    flops_per_iter: float = 0.0
    bytes_per_iter: float = 0.0


@dataclass
class BenchResult:
    config: BenchConfig
    raw_nanos: list[float]
    stats: "Statistics" = None

    def __post_init__(self):
        if self.stats is None:
            self.stats = Statistics.compute(self.raw_nanos)

    def mean_nanos(self) -> float:
        return self.stats.mean

    def throughput_per_s(self) -> float:
        return self.config.batch_size / (self.stats.mean * 1e-9) if self.stats.mean > 0 else 0.0

    def tflops(self) -> float:
        return self.config.flops_per_iter / (self.stats.mean * 1e-9) / 1e12 if self.stats.mean > 0 else 0.0

    def gbps(self) -> float:
        return self.config.bytes_per_iter / (self.stats.mean * 1e-9) / 1e9 if self.stats.mean > 0 else 0.0


def percentile_sorted(sorted_vals: list[float], p: float) -> float:
    """Linear interpolation between closest ranks, p in [0, 100]."""
    if not sorted_vals:
        return 0.0
    k = (len(sorted_vals) - 1) * p / 100.0
    lo, hi = math.floor(k), math.ceil(k)
    return sorted_vals[lo] + (sorted_vals[hi] - sorted_vals[lo]) * (k - lo)


@dataclass
class Statistics:
    count: int = 0
    min: float = 0.0
    max: float = 0.0
    sum: float = 0.0
    mean: float = 0.0
    median: float = 0.0
    mode: float | None = None
    variance: float = 0.0
    std_dev: float = 0.0
    skewness: float = 0.0
    kurtosis: float = 0.0
    p25: float = 0.0
    p50: float = 0.0
    p75: float = 0.0
    p90: float = 0.0
    p95: float = 0.0
    p99: float = 0.0
    p999: float = 0.0
    iqr: float = 0.0
    mad: float = 0.0
    ci_95_lower: float = 0.0
    ci_95_upper: float = 0.0

    @classmethod
    def compute(cls, values) -> "Statistics":
        v = sorted(float(x) for x in values)
        n = len(v)
        if n == 0:
            return cls()
        s = sum(v)
        mean = s / n
        var = sum((x - mean) ** 2 for x in v) / (n - 1) if n > 1 else 0.0
        sd = math.sqrt(var)
        m2 = sum((x - mean) ** 2 for x in v) / n
        skew = (sum((x - mean) ** 3 for x in v) / n) / m2 ** 1.5 if m2 > 0 else 0.0
        kurt = (sum((x - mean) ** 4 for x in v) / n) / m2 ** 2 - 3.0 if m2 > 0 else 0.0
        med = percentile_sorted(v, 50)
        counts = {}
        for x in v:
            counts[x] = counts.get(x, 0) + 1
        top = max(counts.values())
        mode = min(x for x, c in counts.items() if c == top) if top > 1 else None
        mad = percentile_sorted(sorted(abs(x - med) for x in v), 50)
        if n > 1:
            from scipy import stats as st
            half = st.t.ppf(0.975, n - 1) * sd / math.sqrt(n)
        else:
            half = 0.0
        p25, p75 = percentile_sorted(v, 25), percentile_sorted(v, 75)
        return cls(n, v[0], v[-1], s, mean, med, mode, var, sd, skew, kurt, p25, med, p75, percentile_sorted(v, 90),
                   percentile_sorted(v, 95), percentile_sorted(v, 99), percentile_sorted(v, 99.9), p75 - p25, mad,
                   mean - half, mean + half)

    @staticmethod
    def trimmed_mean(values, trim_pct: float) -> float:
        v = sorted(values)
        k = int(len(v) * trim_pct / 100.0)
        core = v[k:len(v) - k] or v
        return sum(core) / len(core)


def _time_once(fn, device) -> float:
    if device is not None and str(device).startswith("cuda"):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) * 1e6
    t0 = time.perf_counter_ns()
    fn()
    return float(time.perf_counter_ns() - t0)


class Runner:
    @staticmethod
    def warmup(config: BenchConfig, fn) -> None:
        for _ in range(config.warmup_iters):
            fn()
        if config.device and str(config.device).startswith("cuda"):
            torch.cuda.synchronize()

    @staticmethod
    def discover_batch_size(target_seconds: float, fn, max_batch: int = 1 << 20) -> int:
        """Doubles the number of calls per sample until one sample takes at least ``target_seconds``."""
        b = 1
        while b < max_batch:
            t0 = time.perf_counter()
            for _ in range(b):
                fn()
            if time.perf_counter() - t0 >= target_seconds:
                break
            b *= 2
        return b

    @staticmethod
    def run_benchmark(config: BenchConfig, fn) -> BenchResult:
        Runner.warmup(config, fn)
        return BenchResult(config, [_time_once(fn, config.device) for _ in range(config.measure_iters)])

    @staticmethod
    def run_sweep(name: str, params, make_fn, **cfg) -> list:
        out = []
        for p in params:
            fn = make_fn(p)
            out.append((p, Runner.run_benchmark(BenchConfig(f"{name}[{p}]", **cfg), fn)))
        return out

    @staticmethod
    def bench_iter(iters: int, fn) -> float:
        t0 = time.perf_counter_ns()
        for _ in range(iters):
            fn()
        return float(time.perf_counter_ns() - t0)


# ------------------------------------------------------------------ comparison
def welch_t_test(a, b):
    """(t, two-sided p) for H0: equal means, unequal variances; t > 0 when mean(b) > mean(a)."""
    if len(a) < 2 or len(b) < 2:
        return 0.0, 1.0
    n1, n2 = len(a), len(b)
    m1, m2 = sum(a) / n1, sum(b) / n2
    v1 = sum((x - m1) ** 2 for x in a) / (n1 - 1)
    v2 = sum((x - m2) ** 2 for x in b) / (n2 - 1)
    se2 = v1 / n1 + v2 / n2
    if se2 <= 1e-24:
        return 0.0, 1.0 if m1 == m2 else 0.0
    t = (m2 - m1) / math.sqrt(se2)
    df = se2 ** 2 / ((v1 / n1) ** 2 / (n1 - 1) + (v2 / n2) ** 2 / (n2 - 1))
    from scipy import stats as st
    return t, float(min(1.0, max(0.0, 2 * st.t.sf(abs(t), df))))


@dataclass
class ComparisonResult:
    name: str
    base_mean: float
    target_mean: float
    speedup_ratio: float
    percent_change: float
    p_value: float
    is_significant: bool
    verdict: str  # "improvement" | "regression" | "no_change"


def compare_runs(base: BenchResult, target: BenchResult, alpha: float = 0.05) -> ComparisonResult:
    bm, tm = base.mean_nanos(), target.mean_nanos()
    pct = (tm - bm) / bm * 100 if bm > 0 else 0.0
    _, p = welch_t_test(base.raw_nanos, target.raw_nanos)
    sig = p < alpha
    verdict = "no_change"
    if sig and pct < -1.0:
        verdict = "improvement"
    elif sig and pct > 1.0:
        verdict = "regression"
    return ComparisonResult(target.config.name, bm, tm, bm / tm if tm > 0 else 1.0, pct, p, sig, verdict)


class BaselineStore:
    """Named results, persisted as JSON; ``evaluate_regressions`` raises when a significant
    regression exceeds the threshold."""

    def __init__(self, path: str | None = None):
        self.path = path
        self.results: dict[str, BenchResult] = {}
        if path and os.path.exists(path):
            with open(path) as f:
                for name, d in json.load(f).items():
                    self.results[name] = BenchResult(BenchConfig(**d["config"]), d["raw_nanos"])

    def add(self, r: BenchResult) -> None:
        self.results[r.config.name] = r

    def get(self, name: str):
        return self.results.get(name)

    def save(self, path: str | None = None) -> None:
        with open(path or self.path, "w") as f:
            json.dump({k: {"config": asdict(r.config), "raw_nanos": r.raw_nanos} for k, r in self.results.items()}, f)

    def evaluate_regressions(self, current, max_regression_pct: float = 5.0):
        comps, fails = [], []
        for r in current:
            base = self.get(r.config.name)
            if base is None:
                continue
            c = compare_runs(base, r)
            if c.verdict == "regression" and c.percent_change > max_regression_pct:
                fails.append(f"benchmark '{c.name}' regressed by {c.percent_change:.2f}% "
                             f"(threshold {max_regression_pct:.2f}%)")
            comps.append(c)
        if fails:
            raise RuntimeError("; ".join(fails))
        return comps


# ------------------------------------------------------------------ hardware / energy / histogram
@dataclass
class HardwareInfo:
    cpu: str = ""
    cpu_count: int = 0
    os: str = ""
    python: str = ""
    torch: str = ""
    gpus: list = field(default_factory=list)

    @classmethod
    def probe(cls) -> "HardwareInfo":
        gpus = []
        if torch.cuda.is_available():
            for i in range(torch.cuda.device_count()):
                p = torch.cuda.get_device_properties(i)
                gpus.append({"name": p.name, "sm_count": p.multi_processor_count, "memory_gb": p.total_memory / 2 ** 30,
                             "capability": f"{p.major}.{p.minor}"})
        return cls(platform.processor() or platform.machine(), os.cpu_count() or 0, platform.platform(),
                   platform.python_version(), torch.__version__, gpus)


def read_gpu_power_watts(index: int = 0):
    """Board power from NVML (a read-only query); None when NVML is not readable."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(index)
        return pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
    except Exception:
        return None


class EnergyEstimator:
    @staticmethod
    def estimate_joules(seconds: float, watts: float) -> float:
        return seconds * watts

    @staticmethod
    def compute_efficiency_gflops_per_watt(gflops: float, watts: float) -> float:
        return gflops / watts if watts > 0 else 0.0


class LogHistogram:
    """Latency histogram with 4 sub-buckets per power of two (nanoseconds); percentiles are accurate
    to about 19 %."""

    SUB = 4

    def __init__(self):
        self.buckets: dict[int, int] = {}
        self.n, self.lo, self.hi = 0, None, None

    def _idx(self, v: int) -> int:
        if v <= 0:
            return 0
        e = v.bit_length() - 1
        frac = (v - (1 << e)) * self.SUB >> e if e > 0 else 0
        return e * self.SUB + frac + 1

    def _value(self, idx: int) -> float:
        if idx == 0:
            return 0.0
        e, frac = divmod(idx - 1, self.SUB)
        return (1 << e) * (1 + (frac + 0.5) / self.SUB)

    def record(self, nanos: int) -> None:
        i = self._idx(int(nanos))
        self.buckets[i] = self.buckets.get(i, 0) + 1
        self.n += 1
        self.lo = nanos if self.lo is None else min(self.lo, nanos)
        self.hi = nanos if self.hi is None else max(self.hi, nanos)

    def count(self) -> int:
        return self.n

    def min(self):
        return self.lo or 0

    def max(self):
        return self.hi or 0

    def percentile(self, p: float) -> float:
        if not self.n:
            return 0.0
        target = max(1, math.ceil(self.n * p / 100.0))
        acc = 0
        for i in sorted(self.buckets):
            acc += self.buckets[i]
            if acc >= target:
                return min(max(self._value(i), self.lo), self.hi)
        return float(self.hi)


# ------------------------------------------------------------------ reports / exporters
def _rows(results):
    for r in results:
        s = r.stats
        yield r.config.name, s.mean / 1e6, s.p50 / 1e6, s.p95 / 1e6, s.p99 / 1e6, s.std_dev / 1e6, s.count


def format_console(results) -> str:
    lines = [f"{'benchmark':40s} {'mean ms':>10s} {'p50':>10s} {'p95':>10s} {'p99':>10s} {'std':>9s} {'n':>5s}"]
    for name, m, p50, p95, p99, sd, n in _rows(results):
        lines.append(f"{name:40s} {m:10.4f} {p50:10.4f} {p95:10.4f} {p99:10.4f} {sd:9.4f} {n:5d}")
    return "\n".join(lines)


def format_markdown(results) -> str:
    out = ["| benchmark | mean ms | p50 ms | p95 ms | p99 ms | std ms | n |", "|---|---|---|---|---|---|---|"]
    for name, m, p50, p95, p99, sd, n in _rows(results):
        out.append(f"| {name} | {m:.4f} | {p50:.4f} | {p95:.4f} | {p99:.4f} | {sd:.4f} | {n} |")
    return "\n".join(out)


def format_csv(results) -> str:
    out = ["name,mean_ms,p50_ms,p95_ms,p99_ms,std_ms,n"]
    for row in _rows(results):
        out.append(",".join([row[0]] + [f"{x:.6f}" for x in row[1:6]] + [str(row[6])]))
    return "\n".join(out)


def format_json(results) -> str:
    return json.dumps([{"name": r.config.name, "stats": asdict(r.stats), "throughput_per_s": r.throughput_per_s(),
                        "tflops": r.tflops(), "gbps": r.gbps()} for r in results], indent=1)


def format_html(results) -> str:
    rows = "".join(f"<tr><td>{n}</td><td>{m:.4f}</td><td>{p50:.4f}</td><td>{p95:.4f}</td><td>{p99:.4f}</td></tr>"
                   for n, m, p50, p95, p99, _, _ in _rows(results))
    return ("<table><tr><th>benchmark</th><th>mean ms</th><th>p50</th><th>p95</th><th>p99</th></tr>" + rows +
            "</table>")


def _metric_name(s: str) -> str:
    return "".join(c if c.isalnum() else "_" for c in s)


class PrometheusExporter:
    @staticmethod
    def export(results) -> str:
        lines = ["# HELP brain_bench_mean_seconds Mean time per iteration", "# TYPE brain_bench_mean_seconds gauge"]
        for r in results:
            lines.append(f'brain_bench_mean_seconds{{name="{_metric_name(r.config.name)}"}} {r.stats.mean * 1e-9:.9g}')
        lines += ["# TYPE brain_bench_p99_seconds gauge"]
        for r in results:
            lines.append(f'brain_bench_p99_seconds{{name="{_metric_name(r.config.name)}"}} {r.stats.p99 * 1e-9:.9g}')
        return "\n".join(lines) + "\n"


class OpenTelemetryExporter:
    @staticmethod
    def export(results) -> str:
        now = time.time_ns()
        return json.dumps({"resourceMetrics": [{"scopeMetrics": [{"metrics": [
            {"name": "brain.bench.mean_ns", "gauge": {"dataPoints": [
                {"asDouble": r.stats.mean, "timeUnixNano": now,
                 "attributes": [{"key": "name", "value": {"stringValue": r.config.name}}]} for r in results]}}]}]}]})


# ------------------------------------------------------------------ kernel suite
class KernelSuite:
    """Times the framework's kernels (GEMM, RMSNorm, softmax cross-entropy) at a given size on the GPU,
    or torch's on the CPU, and reports TFLOP/s or GB/s."""

    @staticmethod
    def run(n: int = 2048, iters: int = 10, device: str | None = None):
        device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        cuda = device.startswith("cuda")
        dt = torch.bfloat16 if cuda else torch.float32
        a = torch.randn(n, n, device=device, dtype=dt)
        b = torch.randn(n, n, device=device, dtype=dt)
        w = torch.ones(n, device=device, dtype=dt)
        labels = torch.randint(0, n, (n,), device=device)
        if cuda:
            from .. import ops
            mm = lambda: ops.gemm(a, b)  # noqa: E731
            norm = lambda: ops.rms_norm(a, w, 1e-6)  # noqa: E731
            ce = lambda: ops.cross_entropy(a, labels)  # noqa: E731
        else:
            mm = lambda: a @ b.t()  # noqa: E731
            norm = lambda: a * torch.rsqrt(a.pow(2).mean(-1, keepdim=True) + 1e-6) * w  # noqa: E731
            ce = lambda: torch.nn.functional.cross_entropy(a, labels)  # noqa: E731
        es = a.element_size()
        cfgs = [BenchConfig("gemm", 2, iters, device=device, flops_per_iter=2.0 * n ** 3),
                BenchConfig("rms_norm", 2, iters, device=device, bytes_per_iter=2.0 * n * n * es),
                BenchConfig("softmax_cross_entropy", 2, iters, device=device, bytes_per_iter=1.0 * n * n * es)]
        return [Runner.run_benchmark(c, f) for c, f in zip(cfgs, (mm, norm, ce))]


# ------------------------------------------------------------------ suites, timers, formatting
# Reference: crates/brain-benchmark/src/suite.rs (BenchmarkSuite::run_all / run_filtered),
# impl.rs (FnBenchmark::from_fn, flop_count), timer.rs (BenchTimer start_new / elapsed_*, calibrate_timer_overhead),
# utils.rs (format_gflops, format_throughput, round_places), hardware.rs (estimate_memory_bandwidth_gbps),
# memory_bench.rs (get_peak_rss_kb).

class FnBenchmark:
    """A named callable with its work per call; ``run`` times it with ``Runner.run_benchmark``."""

    def __init__(self, name: str, fn, flops: float = 0.0, nbytes: float = 0.0, device=None, warmup: int = 3,
                 iters: int = 20, tags=()):
        self.name, self.fn, self.tags = name, fn, set(tags)
        self.config = BenchConfig(name, warmup, iters, 1, device, flops, nbytes)

    @classmethod
    def from_fn(cls, name: str, fn, **kw) -> "FnBenchmark":
        return cls(name, fn, **kw)

    def flop_count(self) -> float:
        return self.config.flops_per_iter

    def run(self) -> BenchResult:
        return Runner.run_benchmark(self.config, self.fn)


class BenchmarkSuite:
    def __init__(self, name: str = "suite"):
        self.name, self.benchmarks = name, []

    def add(self, bench: FnBenchmark) -> "BenchmarkSuite":
        self.benchmarks.append(bench)
        return self

    def run_all(self) -> dict:
        return {b.name: b.run() for b in self.benchmarks}

    def run_filtered(self, pattern: str = "", tag: str | None = None) -> dict:
        return {b.name: b.run() for b in self.benchmarks
                if pattern in b.name and (tag is None or tag in b.tags)}


class BenchTimer:
    """Wall-clock stopwatch (perf_counter_ns)."""

    def __init__(self):
        self._t0, self._t1 = None, None

    @classmethod
    def start_new(cls) -> "BenchTimer":
        t = cls()
        t.start()
        return t

    def start(self):
        self._t0, self._t1 = time.perf_counter_ns(), None

    def stop(self):
        self._t1 = time.perf_counter_ns()

    def is_running(self) -> bool:
        return self._t0 is not None and self._t1 is None

    def elapsed_nanos(self) -> int:
        end = self._t1 if self._t1 is not None else time.perf_counter_ns()
        return end - self._t0

    def elapsed_micros(self) -> float:
        return self.elapsed_nanos() / 1e3

    def elapsed_millis(self) -> float:
        return self.elapsed_nanos() / 1e6

    def elapsed_secs(self) -> float:
        return self.elapsed_nanos() / 1e9


def calibrate_timer_overhead(samples: int = 1000) -> float:
    """Median cost in ns of reading the clock twice back to back."""
    d = []
    for _ in range(samples):
        a = time.perf_counter_ns()
        b = time.perf_counter_ns()
        d.append(b - a)
    d.sort()
    return float(d[len(d) // 2])


def round_places(x: float, places: int) -> float:
    return round(x, places)


def format_gflops(flops: float, seconds: float) -> str:
    v = flops / seconds / 1e9 if seconds > 0 else 0.0
    return f"{v / 1e3:.2f} TFLOP/s" if v >= 1e3 else f"{v:.2f} GFLOP/s"


def format_throughput(items: float, seconds: float, unit: str = "items") -> str:
    v = items / seconds if seconds > 0 else 0.0
    for s, f in (("G", 1e9), ("M", 1e6), ("k", 1e3)):
        if v >= f:
            return f"{v / f:.2f} {s}{unit}/s"
    return f"{v:.2f} {unit}/s"


def estimate_memory_bandwidth_gbps(nbytes: int = 1 << 28, device=None, iters: int = 5) -> float:
    """Copy bandwidth (read + write bytes per second) of one device buffer into another."""
    dev = torch.device(device) if device is not None else torch.device("cuda" if torch.cuda.is_available() else "cpu")
    a = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    b = torch.empty_like(a)
    b.copy_(a)
    if dev.type == "cuda":
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(iters):
            b.copy_(a)
        e.record()
        torch.cuda.synchronize()
        sec = s.elapsed_time(e) / 1e3
    else:
        t0 = time.perf_counter()
        for _ in range(iters):
            b.copy_(a)
        sec = time.perf_counter() - t0
    return 2.0 * nbytes * iters / sec / 1e9


def get_peak_rss_kb() -> int:
    import resource
    return int(resource.getrusage(resource.RUSAGE_SELF).ru_maxrss)
