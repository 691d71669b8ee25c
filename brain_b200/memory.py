"""Memory management on the device: allocation statistics, a bump arena that carves aligned tensors out
of one allocation, a size-binned pool of reusable buffers, and a view of the CUDA caching allocator.

Reference: crates/brain-core/src/memory.rs (``AlignedBuffer`` :179-340, ``AllocationStats`` :415-480,
``MemoryBlock`` / ``SimplePool`` :483-600, ``BinnedMemoryPool``, ``MemoryArena``). The reference pools
host memory for its CPU tensors; here the same roles serve GPU workspaces: an arena gives the kernels
of one step their scratch from a single up-front allocation (no allocator calls inside a CUDA graph
capture, and addresses that do not move between replays), and the binned pool recycles buffers by
power-of-two size class. Every carve is aligned (256 bytes by default, enough for TMA and vector
loads). The communication buffers have their own symmetric allocator (``parallel.symm``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


def is_aligned(t: torch.Tensor, alignment: int = 16) -> bool:
    return t.data_ptr() % alignment == 0


def strides_row_major(shape) -> list[int]:
    out, acc = [], 1
    for d in reversed(list(shape)):
        out.append(acc)
        acc *= d
    return out[::-1]


@dataclass
class AllocationStats:
    allocations: int = 0
    deallocations: int = 0
    bytes_in_use: int = 0
    peak_bytes: int = 0
    total_allocated: int = 0

    def record_allocation(self, size: int) -> None:
        self.allocations += 1
        self.bytes_in_use += size
        self.total_allocated += size
        self.peak_bytes = max(self.peak_bytes, self.bytes_in_use)

    def record_deallocation(self, size: int) -> None:
        self.deallocations += 1
        self.bytes_in_use -= size

    def fragmentation_ratio(self, reserved: int) -> float:
        """Share of reserved bytes not in use."""
        return 1.0 - self.bytes_in_use / reserved if reserved > 0 else 0.0


def aligned_empty(shape, dtype=torch.float32, device=None, alignment: int = 256) -> torch.Tensor:
    """A tensor whose first element is ``alignment``-byte aligned (over-allocates and offsets)."""
    esz = torch.empty((), dtype=dtype).element_size()
    n = 1
    for d in shape:
        n *= d
    raw = torch.empty(n * esz + alignment, dtype=torch.uint8, device=device)
    off = (-raw.data_ptr()) % alignment
    return raw[off:off + n * esz].view(dtype).view(tuple(shape))


class MemoryArena:
    """Bump allocator over one device buffer. ``alloc`` returns aligned views; ``reset`` frees all
    of them at once (the caller guarantees no kernel still uses them). ``mark`` / ``release_to`` give
    stack-like scopes."""

    def __init__(self, capacity_bytes: int, device=None, alignment: int = 256):
        self.alignment = alignment
        self.buf = aligned_empty((capacity_bytes,), torch.uint8, device, alignment)
        self.capacity = capacity_bytes
        self.offset = 0
        self.stats = AllocationStats()

    def alloc(self, shape, dtype=torch.float32) -> torch.Tensor:
        esz = torch.empty((), dtype=dtype).element_size()
        n = 1
        for d in shape:
            n *= d
        start = -(-self.offset // self.alignment) * self.alignment
        end = start + n * esz
        if end > self.capacity:
            raise MemoryError(f"arena exhausted: need {end - self.offset} bytes at offset {self.offset}, "
                              f"capacity {self.capacity}")
        self.offset = end
        self.stats.record_allocation(end - start)
        return self.buf[start:end].view(dtype).view(tuple(shape))

    def mark(self) -> int:
        return self.offset

    def release_to(self, mark: int) -> None:
        self.stats.record_deallocation(self.offset - mark)
        self.offset = mark

    def reset(self) -> None:
        self.release_to(0)

    def used(self) -> int:
        return self.offset


class BinnedMemoryPool:
    """Recycles flat byte buffers by power-of-two size class (minimum ``min_bytes``). ``get`` returns a
    typed view of a pooled buffer; ``put`` gives the buffer back. Buffers never shrink; ``trim`` drops
    the free ones."""

    def __init__(self, device=None, min_bytes: int = 512, alignment: int = 256):
        self.device, self.min_bytes, self.alignment = device, min_bytes, alignment
        self.free: dict[int, list[torch.Tensor]] = {}
        self.stats = AllocationStats()
        self.hits = self.misses = 0

    def _bin(self, nbytes: int) -> int:
        b = self.min_bytes
        while b < nbytes:
            b *= 2
        return b

    def get(self, shape, dtype=torch.float32) -> torch.Tensor:
        esz = torch.empty((), dtype=dtype).element_size()
        n = 1
        for d in shape:
            n *= d
        b = self._bin(n * esz)
        lst = self.free.get(b)
        if lst:
            raw = lst.pop()
            self.hits += 1
        else:
            raw = aligned_empty((b,), torch.uint8, self.device, self.alignment)
            self.misses += 1
        self.stats.record_allocation(b)
        t = raw[:n * esz].view(dtype).view(tuple(shape))
        t._brain_pool_raw = raw
        return t

    def put(self, t: torch.Tensor) -> None:
        raw = getattr(t, "_brain_pool_raw", None)
        if raw is None:
            raise ValueError("tensor was not allocated by this pool")
        self.free.setdefault(raw.numel(), []).append(raw)
        self.stats.record_deallocation(raw.numel())
        del t._brain_pool_raw

    def trim(self) -> int:
        freed = sum(r.numel() for lst in self.free.values() for r in lst)
        self.free.clear()
        return freed


def device_memory_summary(device=None) -> dict:
    """Current / peak allocated and reserved bytes of torch's caching allocator on ``device``."""
    if not torch.cuda.is_available():
        return {}
    s = torch.cuda.memory_stats(device)
    free, total = torch.cuda.mem_get_info(device)
    return {"allocated": s.get("allocated_bytes.all.current", 0), "peak_allocated": s.get("allocated_bytes.all.peak", 0),
            "reserved": s.get("reserved_bytes.all.current", 0), "free": free, "total": total}


# ------------------------------------------------------------------ arena scopes, leak tracking, static planning
# Reference: crates/brain-core/src/memory.rs:752-870 (ArenaCheckpoint, alloc_slice, remaining_bytes),
# :876-975 (MemoryTracker: tagged records, current / peak bytes, leak listing), :977-1060 (TensorLifetime,
# MemoryPlanner: peak of overlapping lifetimes and per-tensor offsets), :84-160 (MemoryFormat strides).

@dataclass(frozen=True)
class ArenaCheckpoint:
    offset: int


def _arena_checkpoint(self) -> ArenaCheckpoint:
    return ArenaCheckpoint(self.offset)


def _arena_rewind(self, cp: ArenaCheckpoint) -> None:
    if cp.offset > self.offset:
        raise ValueError(f"checkpoint {cp.offset} is past the current offset {self.offset}")
    self.release_to(cp.offset)


MemoryArena.checkpoint = _arena_checkpoint
MemoryArena.rewind = _arena_rewind
MemoryArena.alloc_slice = lambda self, count, dtype=torch.float32: self.alloc((count,), dtype)
MemoryArena.remaining_bytes = lambda self: self.capacity - self.offset


@dataclass
class AllocationRecord:
    id: int
    size: int
    tag: str
    tick: int = 0


class MemoryTracker:
    """Thread-safe registry of live allocations by id and tag: current and peak bytes, and the records
    still alive (``find_leaks``) when a scope ends."""

    def __init__(self):
        import threading
        self._lock = threading.Lock()
        self._records: dict[int, AllocationRecord] = {}
        self._next, self._cur, self._peak, self._tick = 1, 0, 0, 0

    def track(self, size: int, tag: str = "") -> int:
        with self._lock:
            rid = self._next
            self._next += 1
            self._tick += 1
            self._cur += size
            self._peak = max(self._peak, self._cur)
            self._records[rid] = AllocationRecord(rid, size, tag, self._tick)
            return rid

    def track_tensor(self, t: torch.Tensor, tag: str = "") -> int:
        return self.track(t.numel() * t.element_size(), tag)

    def untrack(self, rid: int) -> AllocationRecord | None:
        with self._lock:
            rec = self._records.pop(rid, None)
            if rec is not None:
                self._cur -= rec.size
            return rec

    def active_count(self) -> int:
        return len(self._records)

    def current_bytes(self) -> int:
        return self._cur

    def peak_bytes(self) -> int:
        return self._peak

    def find_leaks(self) -> list[AllocationRecord]:
        with self._lock:
            return sorted(self._records.values(), key=lambda r: r.id)

    def reset(self) -> None:
        with self._lock:
            self._records.clear()
            self._cur = self._peak = 0


@dataclass(frozen=True)
class TensorLifetime:
    start_step: int
    end_step: int  # inclusive
    size_bytes: int


class MemoryPlanner:
    """Static placement of step-scoped buffers in one arena (the workspace of a captured CUDA graph).

    ``compute_peak_memory`` is the largest sum of sizes alive at one step (a sweep over lifetime
    boundaries). ``plan_offsets`` places tensors largest first, each at the lowest ``alignment``-aligned
    offset that does not overlap any already placed tensor whose lifetime intersects its own (greedy by
    size, the arena planners' usual heuristic; it packs tighter than placing in insertion order).
    ``materialize`` carves the planned views out of one allocation."""

    def __init__(self, alignment: int = 256):
        self.lifetimes: list[TensorLifetime] = []
        self.alignment = alignment

    def add_tensor(self, start_step: int, end_step: int, size_bytes: int) -> int:
        if end_step < start_step:
            raise ValueError("end_step must be >= start_step")
        self.lifetimes.append(TensorLifetime(start_step, end_step, size_bytes))
        return len(self.lifetimes) - 1

    def compute_peak_memory(self) -> int:
        events: dict[int, int] = {}
        for lt in self.lifetimes:
            events[lt.start_step] = events.get(lt.start_step, 0) + lt.size_bytes
            events[lt.end_step + 1] = events.get(lt.end_step + 1, 0) - lt.size_bytes
        cur = peak = 0
        for step in sorted(events):
            cur += events[step]
            peak = max(peak, cur)
        return peak

    def plan_offsets(self) -> list[int]:
        a = self.alignment
        order = sorted(range(len(self.lifetimes)), key=lambda i: (-self.lifetimes[i].size_bytes, i))
        placed: list[tuple[int, int, TensorLifetime]] = []  # (offset, end, lifetime)
        offsets = [0] * len(self.lifetimes)
        for i in order:
            lt = self.lifetimes[i]
            busy = sorted((o, e) for o, e, other in placed
                          if not (lt.end_step < other.start_step or lt.start_step > other.end_step))
            off = 0
            for o, e in busy:
                if off + lt.size_bytes <= o:
                    break
                off = max(off, -(-e // a) * a)
            offsets[i] = off
            placed.append((off, off + lt.size_bytes, lt))
        return offsets

    def arena_bytes(self, offsets: list[int] | None = None) -> int:
        offsets = self.plan_offsets() if offsets is None else offsets
        return max((o + lt.size_bytes for o, lt in zip(offsets, self.lifetimes)), default=0)

    def materialize(self, device=None) -> tuple[torch.Tensor, list[torch.Tensor]]:
        """(arena, byte views in add order), each view at its planned offset."""
        offs = self.plan_offsets()
        arena = aligned_empty((max(self.arena_bytes(offs), 1),), torch.uint8, device, self.alignment)
        return arena, [arena[o:o + lt.size_bytes] for o, lt in zip(offs, self.lifetimes)]


class MemoryFormat:
    """Element strides of a layout: contiguous / channels_first (row-major), channels_last (NHWC order
    for a 4-D NCHW shape), blocked (2-D, rows of ``block_size``-element blocks), sparse (none), packed."""
    CONTIGUOUS, CHANNELS_FIRST, CHANNELS_LAST, BLOCKED, SPARSE, PACKED = (
        "contiguous", "channels_first", "channels_last", "blocked", "sparse", "packed")

    def __init__(self, kind: str = "contiguous", block_size: int = 0):
        self.kind, self.block_size = kind, block_size

    def strides(self, shape) -> list[int]:
        shape = list(shape)
        if self.kind == self.CHANNELS_LAST and len(shape) == 4:
            _, c, h, w = shape
            return [h * w * c, 1, w * c, c]
        if self.kind == self.BLOCKED and len(shape) == 2:
            return [shape[1] * self.block_size, self.block_size]
        if self.kind == self.SPARSE:
            return []
        return strides_row_major(shape)

    def is_dense(self) -> bool:
        return self.kind in (self.CONTIGUOUS, self.CHANNELS_FIRST, self.CHANNELS_LAST)

    def __str__(self):
        return f"blocked({self.block_size})" if self.kind == self.BLOCKED else self.kind
