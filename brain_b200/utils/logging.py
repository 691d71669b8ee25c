"""Logging with rank prefixes and JSON output (reference brain-utils log: StandardLogger, ConsoleSink,
RingBufferSink, JsonFormatter, crates/brain-utils/src/log/mod.rs:18-150)."""
from __future__ import annotations

import collections
import json
import logging
import os
import sys
import time


def _rank() -> tuple[int, int]:
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


class RankFormatter(logging.Formatter):
    def format(self, record):
        r, w = _rank()
        return f"[Rank {r}/{w}] {time.strftime('%H:%M:%S')} {record.levelname:5s} {record.name}: {record.getMessage()}"


class JsonFormatter(logging.Formatter):
    def format(self, record):
        r, w = _rank()
        return json.dumps({"ts": record.created, "level": record.levelname, "logger": record.name, "rank": r,
                           "world": w, "msg": record.getMessage()})


class RingBufferHandler(logging.Handler):
    """Keeps the last ``capacity`` formatted records in memory (RingBufferSink)."""

    def __init__(self, capacity: int = 1000):
        super().__init__()
        self.buffer = collections.deque(maxlen=capacity)

    def emit(self, record):
        self.buffer.append(self.format(record))


def get_logger(name: str = "brain", level: int = logging.INFO, json_output: bool = False,
               stream=sys.stderr, master_only: bool = False) -> logging.Logger:
    log = logging.getLogger(name)
    if not log.handlers:
        h = logging.StreamHandler(stream)
        h.setFormatter(JsonFormatter() if json_output else RankFormatter())
        log.addHandler(h)
        log.propagate = False
    log.setLevel(level if (not master_only or _rank()[0] == 0) else logging.WARNING)
    return log


StandardLogger = get_logger
