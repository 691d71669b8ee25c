"""Arena scopes, allocation tracking and the static memory planner."""
import random

import pytest
import torch

from brain_b200.memory import (MemoryArena, MemoryTracker, MemoryPlanner, MemoryFormat, ArenaCheckpoint)


def test_arena_checkpoint_rewind():
    a = MemoryArena(1 << 16)
    x = a.alloc((10,), torch.float32)
    cp = a.checkpoint()
    assert isinstance(cp, ArenaCheckpoint)
    a.alloc_slice(100, torch.float16)
    assert a.remaining_bytes() < (1 << 16) - 256
    a.rewind(cp)
    assert a.used() == cp.offset and x.numel() == 10
    with pytest.raises(ValueError):
        a.rewind(ArenaCheckpoint(1 << 15))


def test_memory_tracker_leaks_and_peak():
    t = MemoryTracker()
    a = t.track(100, "a")
    b = t.track(50, "b")
    c = t.track_tensor(torch.zeros(4, 4), "c")
    assert t.current_bytes() == 214 and t.peak_bytes() == 214 and t.active_count() == 3
    assert t.untrack(a).tag == "a" and t.untrack(a) is None
    t.untrack(c)
    assert t.current_bytes() == 50 and t.peak_bytes() == 214
    assert [r.tag for r in t.find_leaks()] == ["b"] and b == t.find_leaks()[0].id
    t.reset()
    assert t.current_bytes() == 0 and t.find_leaks() == []


def _check_plan(p, offs):
    for i, a in enumerate(p.lifetimes):
        assert offs[i] % p.alignment == 0
        for j, b in enumerate(p.lifetimes[:i]):
            live = not (a.end_step < b.start_step or a.start_step > b.end_step)
            mem = not (offs[i] + a.size_bytes <= offs[j] or offs[j] + b.size_bytes <= offs[i])
            assert not (live and mem), (i, j)


def test_planner_peak_and_offsets():
    p = MemoryPlanner(alignment=256)
    p.add_tensor(0, 1, 1024)
    p.add_tensor(1, 2, 2048)
    p.add_tensor(2, 3, 1024)
    p.add_tensor(3, 4, 512)
    assert p.compute_peak_memory() == 3072
    offs = p.plan_offsets()
    _check_plan(p, offs)
    assert p.arena_bytes(offs) == 3072  # tensors 0 and 2 share memory
    random.seed(0)
    q = MemoryPlanner(alignment=256)
    for _ in range(60):
        s = random.randrange(40)
        q.add_tensor(s, s + random.randrange(6), 256 * random.randrange(1, 40))
    offs = q.plan_offsets()
    _check_plan(q, offs)
    assert q.compute_peak_memory() <= q.arena_bytes(offs) <= 1.5 * q.compute_peak_memory()
    arena, views = q.materialize()
    assert len(views) == 60 and views[5].numel() == q.lifetimes[5].size_bytes
    assert MemoryPlanner().compute_peak_memory() == 0 and MemoryPlanner().plan_offsets() == []
    with pytest.raises(ValueError):
        p.add_tensor(3, 2, 10)


def test_memory_format_strides():
    assert MemoryFormat("channels_last").strides([2, 3, 4, 5]) == list(torch.empty(2, 3, 4, 5).to(
        memory_format=torch.channels_last).stride())
    assert MemoryFormat().strides([2, 3]) == [3, 1]
    assert MemoryFormat("blocked", 8).strides([4, 16]) == [128, 8] and str(MemoryFormat("blocked", 8)) == "blocked(8)"
    assert MemoryFormat("sparse").strides([3]) == [] and not MemoryFormat("sparse").is_dense()
