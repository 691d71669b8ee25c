"""Process-level utilities: rate limiting, retries, safe file I/O, directory statistics, formatting and
parsing of sizes and durations, encodings, a small schema validator, versions, system information, a
metrics registry and a timing tree.

Reference: crates/brain-utils/src/utils.rs (TokenBucketRateLimiter, retry_with_backoff, format_*,
parse_size, pad/truncate, shell_quote, random_uuid_lite), io/ (atomic_write_file, append_file,
ensure_dir, unique_temp_path, sanitize_filename, join_safe, normalize_slashes), fs_stats.rs
(FsStats, scan_dir_stats, dir_size, file_count), serialize_helpers.rs (base64, hex), hash.rs
(hash_combine_64), config/schema.rs (SchemaValidator, FieldDef, FieldType, Constraint), version.rs
(Version), env.rs (SystemInfo), metrics_utils.rs (MetricsRegistry, Metric, MetricType), prof/
(TimingTree). The hardware-abstraction layer of the reference (HID, audio and video sources) has no
role on a GPU server and is not reproduced.
"""
from __future__ import annotations

import base64
import os
import platform
import random
import re
import tempfile
import threading
import time
import uuid
from contextlib import contextmanager
from dataclasses import dataclass, field


# ------------------------------------------------------------------------------------------ rate / retry
class TokenBucketRateLimiter:
    """Capacity ``burst`` tokens refilled at ``rate`` per second; ``try_acquire(n)`` takes n tokens if
    available, ``acquire(n)`` waits for them. Thread-safe."""

    def __init__(self, rate: float, burst: float, clock=time.monotonic):
        self.rate, self.cap, self.clock = float(rate), float(burst), clock
        self.tokens, self.t = float(burst), clock()
        self.lock = threading.Lock()

    def _refill(self):
        now = self.clock()
        self.tokens = min(self.cap, self.tokens + (now - self.t) * self.rate)
        self.t = now

    def try_acquire(self, n: float = 1.0) -> bool:
        with self.lock:
            self._refill()
            if self.tokens >= n:
                self.tokens -= n
                return True
            return False

    def acquire(self, n: float = 1.0, sleep=time.sleep) -> None:
        while not self.try_acquire(n):
            with self.lock:
                wait = (n - self.tokens) / self.rate if self.rate > 0 else 0.01
            sleep(max(wait, 1e-4))


def retry_with_backoff(fn, attempts: int = 5, base_delay: float = 0.1, max_delay: float = 5.0, factor: float = 2.0,
                       jitter: float = 0.1, retry_on=(Exception,), sleep=time.sleep, rng=None):
    """Call fn until it succeeds or ``attempts`` are used; delays grow geometrically (capped) with
    +-jitter; the last exception is re-raised."""
    rng = rng or random.Random(0)
    delay = base_delay
    for i in range(attempts):
        try:
            return fn()
        except retry_on:
            if i == attempts - 1:
                raise
            sleep(min(max_delay, delay) * (1 + rng.uniform(-jitter, jitter)))
            delay *= factor


# ------------------------------------------------------------------------------------------ files
def ensure_dir(path: str) -> str:
    os.makedirs(path, exist_ok=True)
    return path


def atomic_write_file(path: str, data, mode: str = "wb") -> None:
    """Write to a temporary file in the same directory, fsync, then rename over the target, so readers
    see either the old or the new contents, never a torn file."""
    d = os.path.dirname(os.path.abspath(path)) or "."
    fd, tmp = tempfile.mkstemp(dir=d, prefix=".tmp-", suffix=os.path.basename(path))
    try:
        with os.fdopen(fd, mode) as f:
            f.write(data)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise


def append_file(path: str, text: str) -> None:
    with open(path, "a", encoding="utf-8") as f:
        f.write(text)


def unique_temp_path(prefix: str = "brain", suffix: str = "", directory: str | None = None) -> str:
    return os.path.join(directory or tempfile.gettempdir(), f"{prefix}-{uuid.uuid4().hex[:12]}{suffix}")


def sanitize_filename(name: str, replacement: str = "_") -> str:
    """Characters outside [A-Za-z0-9._-] replaced; leading dots stripped; never empty."""
    s = re.sub(r"[^A-Za-z0-9._-]", replacement, name).lstrip(".")
    return s or "unnamed"


def normalize_slashes(path: str) -> str:
    return re.sub(r"/+", "/", path.replace("\\", "/"))


def join_safe(root: str, *parts: str) -> str:
    """Join under ``root`` and refuse paths that escape it (.. or absolute components)."""
    full = os.path.realpath(os.path.join(root, *parts))
    base = os.path.realpath(root)
    if os.path.commonpath([full, base]) != base:
        raise ValueError(f"path escapes {root}: {os.path.join(*parts)}")
    return full


@dataclass
class FsStats:
    files: int = 0
    dirs: int = 0
    bytes: int = 0
    largest_file: str = ""
    largest_bytes: int = 0
    by_extension: dict = field(default_factory=dict)


def scan_dir_stats(root: str) -> FsStats:
    st = FsStats()
    for dirpath, dirnames, filenames in os.walk(root):
        st.dirs += len(dirnames)
        for f in filenames:
            p = os.path.join(dirpath, f)
            try:
                n = os.path.getsize(p)
            except OSError:
                continue
            st.files += 1
            st.bytes += n
            ext = os.path.splitext(f)[1].lower() or "<none>"
            st.by_extension[ext] = st.by_extension.get(ext, 0) + 1
            if n > st.largest_bytes:
                st.largest_bytes, st.largest_file = n, p
    return st


def dir_size(root: str) -> int:
    return scan_dir_stats(root).bytes


def file_count(root: str) -> int:
    return scan_dir_stats(root).files


# ------------------------------------------------------------------------------------------ formatting / parsing
_UNITS = {"b": 1, "k": 1000, "kb": 1000, "m": 1000 ** 2, "mb": 1000 ** 2, "g": 1000 ** 3, "gb": 1000 ** 3,
          "t": 1000 ** 4, "tb": 1000 ** 4, "kib": 1024, "mib": 1024 ** 2, "gib": 1024 ** 3, "tib": 1024 ** 4}


def parse_size(text: str) -> int:
    """'512', '4k', '1.5 MB', '2GiB' -> bytes (decimal units for k/M/G/T, binary for KiB/MiB/GiB/TiB)."""
    m = re.fullmatch(r"\s*([0-9]*\.?[0-9]+)\s*([A-Za-z]*)\s*", text)
    if not m:
        raise ValueError(f"cannot parse size: {text!r}")
    unit = m.group(2).lower() or "b"
    if unit not in _UNITS:
        raise ValueError(f"unknown size unit: {m.group(2)!r}")
    return int(round(float(m.group(1)) * _UNITS[unit]))


def format_bytes(n: float, binary: bool = False) -> str:
    base, units = (1024.0, ["B", "KiB", "MiB", "GiB", "TiB", "PiB"]) if binary else (1000.0, ["B", "KB", "MB", "GB", "TB", "PB"])
    v, i = float(n), 0
    while abs(v) >= base and i < len(units) - 1:
        v, i = v / base, i + 1
    return f"{v:.0f} {units[i]}" if i == 0 else f"{v:.2f} {units[i]}"


def format_bytes_binary(n: float) -> str:
    return format_bytes(n, True)


def format_duration(seconds: float) -> str:
    """Human-readable: 850 ns, 12.3 us, 4.56 ms, 1.23 s, 2m 03s, 1h 02m 03s."""
    s = float(seconds)
    if s < 1e-6:
        return f"{s * 1e9:.0f} ns"
    if s < 1e-3:
        return f"{s * 1e6:.1f} us"
    if s < 1.0:
        return f"{s * 1e3:.2f} ms"
    if s < 60:
        return f"{s:.2f} s"
    m, sec = divmod(int(round(s)), 60)
    if m < 60:
        return f"{m}m {sec:02d}s"
    h, m = divmod(m, 60)
    return f"{h}h {m:02d}m {sec:02d}s"


_DUR = {"ns": 1e-9, "us": 1e-6, "ms": 1e-3, "s": 1.0, "m": 60.0, "min": 60.0, "h": 3600.0}


def parse_duration(text: str) -> float:
    """'250ms', '1.5s', '2m', '3h', '1h30m' -> seconds."""
    parts = re.findall(r"([0-9]*\.?[0-9]+)\s*(ns|us|ms|min|s|m|h)", text.strip().lower())
    if not parts or "".join(a + b for a, b in parts) != re.sub(r"\s+", "", text.strip().lower()):
        raise ValueError(f"cannot parse duration: {text!r}")
    return sum(float(v) * _DUR[u] for v, u in parts)


def format_percent(x: float, digits: int = 1) -> str:
    return f"{100.0 * x:.{digits}f}%"


def pad_left(s: str, width: int, fill: str = " ") -> str:
    return s.rjust(width, fill)


def pad_right(s: str, width: int, fill: str = " ") -> str:
    return s.ljust(width, fill)


def truncate_str(s: str, max_len: int, ellipsis: str = "...") -> str:
    return s if len(s) <= max_len else s[:max(max_len - len(ellipsis), 0)] + ellipsis


def shell_quote(s: str) -> str:
    return "''" if not s else s if re.fullmatch(r"[A-Za-z0-9_./=:-]+", s) else "'" + s.replace("'", "'\"'\"'") + "'"


def base64_encode(data: bytes) -> str:
    return base64.b64encode(data).decode()


def base64_decode(text: str) -> bytes:
    return base64.b64decode(text)


def bytes_to_hex(data: bytes) -> str:
    return data.hex()


def hex_to_bytes(text: str) -> bytes:
    return bytes.fromhex(text)


def hash_combine_64(seed: int, value: int) -> int:
    """Mix a 64-bit hash into a seed (the boost-style combine widened to 64 bits)."""
    m = (1 << 64) - 1
    return (seed ^ ((value + 0x9E3779B97F4A7C15 + ((seed << 6) & m) + (seed >> 2)) & m)) & m


def random_uuid_lite(rng=None) -> str:
    r = rng or random
    return "%08x-%04x-4%03x-%04x-%012x" % (r.getrandbits(32), r.getrandbits(16), r.getrandbits(12),
                                          (r.getrandbits(14) | 0x8000), r.getrandbits(48))


def now_ms() -> int:
    return time.time_ns() // 1_000_000


def now_us() -> int:
    return time.time_ns() // 1_000


def now_ns() -> int:
    return time.time_ns()


# ------------------------------------------------------------------------------------------ schema / versions / system
class FieldType:
    INT, FLOAT, BOOL, STR, LIST, DICT = "int", "float", "bool", "str", "list", "dict"


_PYT = {"int": int, "float": (int, float), "bool": bool, "str": str, "list": list, "dict": dict}


@dataclass
class Constraint:
    min: float | None = None
    max: float | None = None
    choices: tuple | None = None
    pattern: str | None = None


@dataclass
class FieldDef:
    name: str
    type: str
    required: bool = True
    default: object = None
    constraint: Constraint | None = None


class SchemaValidator:
    """Checks a configuration mapping against field definitions: presence, type, numeric range, choices,
    regex; fills defaults; rejects unknown keys when ``strict``. Returns (normalised config, errors)."""

    def __init__(self, fields, strict: bool = False):
        self.fields = {f.name: f for f in fields}
        self.strict = strict

    def validate(self, cfg: dict):
        out, errs = {}, []
        for name, f in self.fields.items():
            if name not in cfg:
                if f.required and f.default is None:
                    errs.append(f"missing field {name}")
                elif f.default is not None:
                    out[name] = f.default
                continue
            v = cfg[name]
            t = _PYT[f.type]
            if f.type != FieldType.BOOL and isinstance(v, bool) or not isinstance(v, t):
                errs.append(f"{name}: expected {f.type}, got {type(v).__name__}")
                continue
            c = f.constraint
            if c is not None:
                if c.min is not None and v < c.min:
                    errs.append(f"{name}: {v} < minimum {c.min}")
                if c.max is not None and v > c.max:
                    errs.append(f"{name}: {v} > maximum {c.max}")
                if c.choices is not None and v not in c.choices:
                    errs.append(f"{name}: {v!r} not in {list(c.choices)}")
                if c.pattern is not None and not re.fullmatch(c.pattern, str(v)):
                    errs.append(f"{name}: {v!r} does not match {c.pattern}")
            out[name] = v
        if self.strict:
            errs += [f"unknown field {k}" for k in cfg if k not in self.fields]
        else:
            out.update({k: v for k, v in cfg.items() if k not in self.fields})
        return out, errs


@dataclass(order=True, frozen=True)
class Version:
    major: int
    minor: int = 0
    patch: int = 0

    @classmethod
    def parse(cls, text: str) -> "Version":
        m = re.fullmatch(r"\s*v?(\d+)(?:\.(\d+))?(?:\.(\d+))?.*", text)
        if not m:
            raise ValueError(f"not a version: {text!r}")
        return cls(int(m.group(1)), int(m.group(2) or 0), int(m.group(3) or 0))

    def is_compatible(self, other: "Version") -> bool:
        """Same major version (and, for 0.x, the same minor), semver-style."""
        return self.major == other.major and (self.major > 0 or self.minor == other.minor)

    def __str__(self):
        return f"{self.major}.{self.minor}.{self.patch}"


@dataclass
class SystemInfo:
    os: str
    python: str
    cpu_count: int
    hostname: str
    torch: str
    cuda_devices: list

    @classmethod
    def collect(cls) -> "SystemInfo":
        import torch
        devs = []
        if torch.cuda.is_available():
            for i in range(torch.cuda.device_count()):
                p = torch.cuda.get_device_properties(i)
                devs.append({"name": p.name, "memory_gib": round(p.total_memory / 2 ** 30, 1),
                             "sms": p.multi_processor_count, "cc": f"{p.major}.{p.minor}"})
        return cls(platform.platform(), platform.python_version(), os.cpu_count() or 1, platform.node(),
                   torch.__version__, devs)


# ------------------------------------------------------------------------------------------ metrics / timing
class MetricType:
    COUNTER, GAUGE, HISTOGRAM = "counter", "gauge", "histogram"


@dataclass
class Metric:
    name: str
    type: str
    value: float = 0.0
    samples: list = field(default_factory=list)


class MetricsRegistry:
    """Named counters (monotone adds), gauges (last value) and histograms (kept samples with
    percentiles); ``snapshot`` returns plain values. Thread-safe."""

    def __init__(self):
        self.metrics: dict[str, Metric] = {}
        self.lock = threading.Lock()

    def _get(self, name, typ):
        m = self.metrics.get(name)
        if m is None:
            m = self.metrics[name] = Metric(name, typ)
        elif m.type != typ:
            raise ValueError(f"{name} is a {m.type}, not a {typ}")
        return m

    def inc(self, name: str, by: float = 1.0) -> None:
        if by < 0:
            raise ValueError("counters only increase")
        with self.lock:
            self._get(name, MetricType.COUNTER).value += by

    def set(self, name: str, value: float) -> None:
        with self.lock:
            self._get(name, MetricType.GAUGE).value = float(value)

    def observe(self, name: str, value: float) -> None:
        with self.lock:
            m = self._get(name, MetricType.HISTOGRAM)
            m.samples.append(float(value))
            m.value += float(value)

    def percentile(self, name: str, q: float) -> float:
        s = sorted(self.metrics[name].samples)
        if not s:
            return 0.0
        k = (len(s) - 1) * q / 100.0
        lo, hi = int(k), min(int(k) + 1, len(s) - 1)
        return s[lo] + (s[hi] - s[lo]) * (k - lo)

    def snapshot(self) -> dict:
        out = {}
        for n, m in self.metrics.items():
            if m.type == MetricType.HISTOGRAM:
                out[n] = {"count": len(m.samples), "sum": m.value, "p50": self.percentile(n, 50),
                          "p99": self.percentile(n, 99)}
            else:
                out[n] = m.value
        return out


class TimingTree:
    """Nested wall-clock sections: ``with tree.section("fwd"):`` blocks nest; ``report`` lists every path
    with its call count and total seconds, children indented under their parent."""

    def __init__(self, clock=time.perf_counter):
        self.clock = clock
        self.totals: dict[tuple, list] = {}
        self.stack: list[str] = []

    @contextmanager
    def section(self, name: str):
        self.stack.append(name)
        key = tuple(self.stack)
        t0 = self.clock()
        try:
            yield
        finally:
            e = self.totals.setdefault(key, [0, 0.0])
            e[0] += 1
            e[1] += self.clock() - t0
            self.stack.pop()

    def report(self) -> str:
        lines = []
        for key in sorted(self.totals):
            n, t = self.totals[key]
            lines.append(f"{'  ' * (len(key) - 1)}{key[-1]}: {n} call(s), {format_duration(t)}")
        return "\n".join(lines)
