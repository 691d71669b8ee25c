"""Operation tape (reference: crates/brain-autograd/src/tape/mod.rs:17-77).

``start_recording`` / ``stop_recording`` / ``with_tape`` record an ``OpRecord`` for every ``Value``
operation executed while recording (op name, input ids, output id, output shape). Like the
reference, the tape is an inspection / IR-export aid: backward does not read it. ``TapePruner``
keeps the records reachable from given outputs; ``TapeFusionPass`` groups elementwise chains that
the kernel layer would fuse.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field

_local = threading.local()


@dataclass
class OpRecord:
    op: str
    inputs: list
    output: int
    shape: tuple


@dataclass
class Tape:
    records: list = field(default_factory=list)

    def __len__(self):
        return len(self.records)

    def ops(self) -> list[str]:
        return [r.op for r in self.records]

    def clear(self):
        self.records.clear()


def _current() -> Tape | None:
    return getattr(_local, "tape", None)


def record(op: str, inputs: list, output: int, shape: tuple) -> None:
    t = _current()
    if t is not None:
        t.records.append(OpRecord(op, list(inputs), output, shape))


def start_recording() -> Tape:
    _local.tape = Tape()
    return _local.tape


def stop_recording() -> Tape | None:
    t = _current()
    _local.tape = None
    return t


def is_recording() -> bool:
    return _current() is not None


def with_tape(fn, *args, **kw):
    """Run fn while recording; returns (result, tape)."""
    prev = _current()
    t = start_recording()
    try:
        out = fn(*args, **kw)
    finally:
        _local.tape = prev
    return out, t


class TapePruner:
    @staticmethod
    def prune(tape: Tape, outputs: list[int]) -> Tape:
        need = set(outputs)
        keep = []
        for r in reversed(tape.records):
            if r.output in need:
                keep.append(r)
                need.update(r.inputs)
        return Tape(list(reversed(keep)))


ELEMENTWISE = {"add", "sub", "mul", "div", "neg", "exp", "log", "relu", "gelu", "silu", "sigmoid", "tanh", "pow"}


class TapeFusionPass:
    @staticmethod
    def groups(tape: Tape) -> list[list[OpRecord]]:
        """Maximal runs of elementwise ops where each consumes the previous output."""
        out, cur = [], []
        for r in tape.records:
            if r.op in ELEMENTWISE and (not cur or cur[-1].output in r.inputs):
                cur.append(r)
            else:
                if len(cur) > 1:
                    out.append(cur)
                cur = [r] if r.op in ELEMENTWISE else []
        if len(cur) > 1:
            out.append(cur)
        return out
