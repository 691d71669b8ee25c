"""Host-side utility APIs with the reference's names: environment lookups, a structured logger
(levels, records with fields, formatters, sinks), CSV reader / writer with quoting, an INI file with
typed getters, a JSON value with typed accessors, and named counter / gauge sets.

Reference: crates/brain-utils/src/env.rs:5-85 (env_get, env_bool accepting true/1/yes/on and
false/0/no/off, env_list splitting on commas, env_prefix_map lower-casing the stripped keys),
log/mod.rs:13-120 (LogLevel, LogRecord, StandardLogger), log/formatters.rs (plain, timestamped,
key=value, JSON), log/sinks.rs (memory, console, multi), io/csv.rs (quoted fields, doubled quotes),
io/ini.rs, io/json.rs, prof/counters.rs (CounterSet, AtomicGauge).
"""
from __future__ import annotations

import csv
import io
import json
import os
import sys
import threading
import time
from dataclasses import dataclass, field

_TRUE = {"true", "1", "yes", "on"}
_FALSE = {"false", "0", "no", "off"}


# ------------------------------------------------------------------ environment
def env_get(key: str) -> str | None:
    return os.environ.get(key)


def env_get_or(key: str, default: str) -> str:
    v = os.environ.get(key)
    return default if v is None else v


def _parse(v, conv, default):
    if v is None:
        return default
    try:
        return conv(v)
    except ValueError:
        return default


def env_i64(key: str, default: int) -> int:
    return _parse(os.environ.get(key), int, default)


def env_f64(key: str, default: float) -> float:
    return _parse(os.environ.get(key), float, default)


def _bool(v, default: bool) -> bool:
    if v is None:
        return default
    s = v.lower()
    return True if s in _TRUE else False if s in _FALSE else default


def env_bool(key: str, default: bool) -> bool:
    return _bool(os.environ.get(key), default)


def env_list(key: str) -> list[str]:
    v = os.environ.get(key)
    return [p.strip() for p in v.split(",") if p.strip()] if v else []


def env_prefix_map(prefix: str) -> dict[str, str]:
    return dict(sorted((k[len(prefix):].lower(), v) for k, v in os.environ.items() if k.startswith(prefix)))


class PrefixEnv:
    """The variables under one prefix, looked up by their lower-cased suffix."""

    def __init__(self, prefix: str):
        self.prefix, self.vars = prefix, env_prefix_map(prefix)

    def get(self, key: str) -> str | None:
        return self.vars.get(key.lower())

    def get_i64(self, key: str, default: int) -> int:
        return _parse(self.get(key), int, default)

    def get_bool(self, key: str, default: bool) -> bool:
        return _bool(self.get(key), default)


# ------------------------------------------------------------------ structured logging
class LogLevel:
    TRACE, DEBUG, INFO, WARN, ERROR, OFF = range(6)
    _NAMES = ("TRACE", "DEBUG", "INFO", "WARN", "ERROR", "OFF")

    @classmethod
    def from_str(cls, s: str) -> int:
        s = s.upper()
        return {"WARNING": cls.WARN, "NONE": cls.OFF}.get(s, cls._NAMES.index(s) if s in cls._NAMES else cls.INFO)

    @classmethod
    def as_str(cls, level: int) -> str:
        return cls._NAMES[level]


@dataclass
class LogRecord:
    level: int
    target: str
    message: str
    timestamp: float = field(default_factory=time.time)
    file: str | None = None
    line: int | None = None
    fields: dict = field(default_factory=dict)

    def with_location(self, file: str, line: int) -> "LogRecord":
        self.file, self.line = file, line
        return self

    def with_field(self, key: str, value) -> "LogRecord":
        self.fields[key] = str(value)
        return self


class PlainFormatter:
    def format(self, r: LogRecord) -> str:
        return f"[{LogLevel.as_str(r.level)}] [{r.target}] {r.message}"


class TimestampedFormatter:
    def __init__(self, show_location: bool = True):
        self.show_location = show_location

    def format(self, r: LogRecord) -> str:
        ts = time.strftime("%Y-%m-%dT%H:%M:%S", time.gmtime(r.timestamp)) + f".{int(r.timestamp * 1000) % 1000:03d}Z"
        loc = f" ({r.file}:{r.line})" if self.show_location and r.file and r.line is not None else ""
        return f"{ts} [{LogLevel.as_str(r.level)}] [{r.target}]{loc} {r.message}"


class KeyValueFormatter:
    def format(self, r: LogRecord) -> str:
        out = f'level={LogLevel.as_str(r.level)} target={r.target} msg="{_esc(r.message)}"'
        return out + "".join(f' {k}="{_esc(v)}"' for k, v in sorted(r.fields.items()))


class JsonLogFormatter:
    def format(self, r: LogRecord) -> str:
        d = {"level": LogLevel.as_str(r.level), "target": r.target, "message": r.message, "timestamp": r.timestamp}
        if r.file:
            d["file"] = r.file
        if r.line is not None:
            d["line"] = r.line
        if r.fields:
            d["fields"] = dict(sorted(r.fields.items()))
        return json.dumps(d)


def _esc(s: str) -> str:
    return str(s).replace('"', '\\"')


class MemorySink:
    """Keeps formatted lines (thread-safe); ``get_messages`` returns a copy."""

    def __init__(self, capacity: int | None = None):
        self._lock, self._lines, self.capacity = threading.Lock(), [], capacity

    def write(self, line: str) -> None:
        with self._lock:
            self._lines.append(line)
            if self.capacity and len(self._lines) > self.capacity:
                del self._lines[0]

    def get_messages(self) -> list[str]:
        with self._lock:
            return list(self._lines)


class ConsoleSink:
    def __init__(self, stream=None):
        self.stream = stream or sys.stderr

    def write(self, line: str) -> None:
        print(line, file=self.stream)


class FileSink:
    def __init__(self, path: str):
        self.path = path

    def write(self, line: str) -> None:
        with open(self.path, "a", encoding="utf-8") as f:
            f.write(line + "\n")


class MultiSink:
    def __init__(self, sinks=()):
        self.sinks = list(sinks)

    def add_sink(self, sink) -> None:
        self.sinks.append(sink)

    def write(self, line: str) -> None:
        for s in self.sinks:
            s.write(line)


class StandardLogger:
    """Level filter -> formatter -> sink. ``log`` returns whether the record was written."""

    def __init__(self, level: int = LogLevel.INFO, sink=None, formatter=None):
        self.level, self.sink, self.formatter = level, sink or ConsoleSink(), formatter or PlainFormatter()

    @classmethod
    def default_console(cls) -> "StandardLogger":
        return cls(LogLevel.INFO, ConsoleSink(), TimestampedFormatter())

    def enabled(self, level: int) -> bool:
        return self.level != LogLevel.OFF and level >= self.level and level != LogLevel.OFF

    def log(self, record: LogRecord) -> bool:
        if not self.enabled(record.level):
            return False
        self.sink.write(self.formatter.format(record))
        return True

    def _at(self, level, target, msg, **fields):
        r = LogRecord(level, target, msg)
        for k, v in fields.items():
            r.with_field(k, v)
        return self.log(r)

    def trace(self, target, msg, **f):
        return self._at(LogLevel.TRACE, target, msg, **f)

    def debug(self, target, msg, **f):
        return self._at(LogLevel.DEBUG, target, msg, **f)

    def info(self, target, msg, **f):
        return self._at(LogLevel.INFO, target, msg, **f)

    def warn(self, target, msg, **f):
        return self._at(LogLevel.WARN, target, msg, **f)

    def error(self, target, msg, **f):
        return self._at(LogLevel.ERROR, target, msg, **f)


def create_record(level: int, target: str, message: str) -> LogRecord:
    return LogRecord(level, target, message)


# ------------------------------------------------------------------ CSV / INI / JSON
@dataclass
class CsvConfig:
    delimiter: str = ","
    quote_char: str = '"'
    has_headers: bool = True


class CsvRecord(list):
    def get(self, i: int):
        return self[i] if 0 <= i < len(self) else None


class CsvReader:
    """Parses quoted fields (a doubled quote is a literal quote); raises on an unterminated quote."""

    def __init__(self, headers, records, config):
        self._headers, self._records, self.config = headers, records, config

    @classmethod
    def parse_str(cls, content: str, config: CsvConfig | None = None) -> "CsvReader":
        c = config or CsvConfig()
        if content.count(c.quote_char) % 2:
            raise ValueError("unterminated quoted CSV field")
        rows = [CsvRecord(r) for r in csv.reader(io.StringIO(content), delimiter=c.delimiter, quotechar=c.quote_char)
                if r]
        headers = list(rows.pop(0)) if c.has_headers and rows else None
        return cls(headers, rows, c)

    def headers(self):
        return self._headers

    def records(self):
        return self._records


class CsvWriter:
    def __init__(self, config: CsvConfig | None = None):
        self.config = config or CsvConfig()
        self._buf = io.StringIO()
        self._w = csv.writer(self._buf, delimiter=self.config.delimiter, quotechar=self.config.quote_char,
                             lineterminator="\n")

    def write_record(self, fields) -> None:
        self._w.writerow([str(f) for f in fields])

    def to_string(self) -> str:
        return self._buf.getvalue()


class IniFile:
    """Sections of key = value lines (``;`` / ``#`` comments); typed getters with defaults."""

    def __init__(self, sections: dict | None = None):
        self.sections = sections or {}

    @classmethod
    def parse(cls, text: str) -> "IniFile":
        sec, cur = {}, "default"
        for raw in text.splitlines():
            line = raw.strip()
            if not line or line[0] in ";#":
                continue
            if line.startswith("[") and line.endswith("]"):
                cur = line[1:-1].strip()
                sec.setdefault(cur, {})
            elif "=" in line:
                k, v = line.split("=", 1)
                sec.setdefault(cur, {})[k.strip()] = v.strip()
        return cls(sec)

    def get(self, section: str, key: str) -> str | None:
        return self.sections.get(section, {}).get(key)

    def get_i64(self, section, key, default: int = 0) -> int:
        return _parse(self.get(section, key), int, default)

    def get_f64(self, section, key, default: float = 0.0) -> float:
        return _parse(self.get(section, key), float, default)

    def get_bool(self, section, key, default: bool = False) -> bool:
        return _bool(self.get(section, key), default)

    def to_string(self) -> str:
        out = []
        for s, kv in self.sections.items():
            out.append(f"[{s}]")
            out += [f"{k} = {v}" for k, v in kv.items()]
            out.append("")
        return "\n".join(out)


class JsonValue:
    """A parsed JSON value with typed accessors that return None on a type mismatch."""

    def __init__(self, value):
        self.value = value

    @classmethod
    def parse(cls, text: str) -> "JsonValue":
        return cls(json.loads(text))

    def as_bool(self):
        return self.value if isinstance(self.value, bool) else None

    def as_f64(self):
        return float(self.value) if isinstance(self.value, (int, float)) and not isinstance(self.value, bool) else None

    def as_str(self):
        return self.value if isinstance(self.value, str) else None

    def as_array(self):
        return [JsonValue(v) for v in self.value] if isinstance(self.value, list) else None

    def as_object(self):
        return {k: JsonValue(v) for k, v in self.value.items()} if isinstance(self.value, dict) else None

    def get(self, key):
        if isinstance(self.value, dict) and key in self.value:
            return JsonValue(self.value[key])
        if isinstance(self.value, list) and isinstance(key, int) and -len(self.value) <= key < len(self.value):
            return JsonValue(self.value[key])
        return None

    def is_null(self) -> bool:
        return self.value is None

    def to_compact_string(self) -> str:
        return json.dumps(self.value, separators=(",", ":"))

    def to_pretty_string(self, indent: int = 2) -> str:
        return json.dumps(self.value, indent=indent)


# ------------------------------------------------------------------ counters
class AtomicGauge:
    def __init__(self, value: float = 0.0):
        self._lock, self._v = threading.Lock(), float(value)

    def set(self, v: float) -> None:
        with self._lock:
            self._v = float(v)

    def add(self, d: float) -> float:
        with self._lock:
            self._v += d
            return self._v

    def get(self) -> float:
        return self._v


class CounterSet:
    """Named integer counters and float gauges created on first use; snapshots are sorted dicts."""

    def __init__(self):
        self._lock = threading.Lock()
        self._c: dict[str, int] = {}
        self._g: dict[str, AtomicGauge] = {}

    def increment(self, name: str, by: int = 1) -> int:
        with self._lock:
            self._c[name] = self._c.get(name, 0) + by
            return self._c[name]

    def get_counter(self, name: str) -> int:
        return self._c.get(name, 0)

    def get_gauge(self, name: str) -> AtomicGauge:
        with self._lock:
            return self._g.setdefault(name, AtomicGauge())

    def snapshot_counters(self) -> dict[str, int]:
        with self._lock:
            return dict(sorted(self._c.items()))

    def snapshot_gauges(self) -> dict[str, float]:
        with self._lock:
            return {k: g.get() for k, g in sorted(self._g.items())}

    def reset_all(self) -> None:
        with self._lock:
            self._c.clear()
            for g in self._g.values():
                g.set(0.0)


def read_file_str(path: str) -> str:
    with open(path, encoding="utf-8") as f:
        return f.read()


def read_file_bytes(path: str) -> bytes:
    with open(path, "rb") as f:
        return f.read()


def delete_file(path: str) -> bool:
    try:
        os.remove(path)
        return True
    except FileNotFoundError:
        return False
