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
