"""Public collectives: ``all_reduce``, ``all_gather``, ``reduce_scatter``, ``broadcast``, ``barrier``.

The reference declares these (crates/brain-distributed/src/collective/mod.rs:18-21,
allreduce.rs:9-121) but only simulates all-reduce in one process. Here they run across processes:
on CUDA tensors with more than one rank they use the in-kernel NVLink backend
(``parallel.symm.NvlinkComm``: P2P loads/stores over NVSwitch); ``backend="nccl"`` selects NCCL;
CPU tensors use Gloo. ``ring_allreduce_simulate`` keeps the reference's in-process algorithm
(pad to p * ceil(n/p), p-1 reduce-scatter steps, p-1 all-gather steps) for tests and teaching.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .comm import NcclComm

_comms: dict = {}


def _world(group=None) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


def get_comm(backend: str | None = None, group=None):
    """The communicator for ``backend`` ("nvlink" default on CUDA, "nccl", "gloo")."""
    key = (backend, id(group))
    c = _comms.get(key)
    if c is None:
        if backend == "nvlink" or (backend is None and torch.cuda.is_available()
                                   and dist.is_initialized() and dist.get_backend(group) == "nccl"):
            from .symm import NvlinkComm
            c = NvlinkComm(group)
        else:
            c = NcclComm(group)
        _comms[key] = c
    return c


def all_reduce(t: torch.Tensor, op: str = "sum", group=None, backend: str | None = None) -> torch.Tensor:
    """In-place all-reduce (sum / mean / max / min)."""
    if _world(group) == 1:
        return t
    if not t.is_cuda:
        if op in ("mean", "avg"):
            _mean_gloo(t, group)
        else:
            NcclComm(group).all_reduce(t, op)
        return t
    return get_comm(backend, group).all_reduce(t, op)


def _mean_gloo(t, group):
    dist.all_reduce(t, group=group)
    t.div_(dist.get_world_size(group))


def reduce_scatter(t: torch.Tensor, group=None, backend: str | None = None, op: str = "sum") -> torch.Tensor:
    """Sum of ``t`` over ranks, returning this rank's 1/world slice (first dim split)."""
    w = _world(group)
    if w == 1:
        return t.clone()
    flat = t.contiguous().view(-1)
    if flat.numel() % w:
        raise ValueError("reduce_scatter needs numel divisible by world size")
    out = torch.empty(flat.numel() // w, device=t.device, dtype=t.dtype)
    if t.is_cuda:
        get_comm(backend, group).reduce_scatter_flat(flat, out, op)
    else:
        NcclComm(group).reduce_scatter_flat(flat, out, op)
    if op in ("mean", "avg"):
        out.div_(w)
    return out.view(t.shape[0] // w, *t.shape[1:]) if t.dim() > 1 and t.shape[0] % w == 0 else out


def all_gather(t: torch.Tensor, group=None, backend: str | None = None) -> torch.Tensor:
    """Concatenation of every rank's ``t`` along a new leading chunk (returns [world * numel])."""
    w = _world(group)
    if w == 1:
        return t.clone().view(-1)
    shard = t.contiguous().view(-1)
    full = torch.empty(shard.numel() * w, device=t.device, dtype=t.dtype)
    if t.is_cuda:
        get_comm(backend, group).all_gather_flat(shard, full)
    else:
        NcclComm(group).all_gather_flat(shard, full)
    return full


def broadcast(t: torch.Tensor, src: int = 0, group=None, backend: str | None = None) -> torch.Tensor:
    if _world(group) == 1:
        return t
    if t.is_cuda:
        return get_comm(backend, group).broadcast(t, src)
    dist.broadcast(t, src, group=group)
    return t


def barrier(group=None) -> None:
    if dist.is_initialized():
        dist.barrier(group)


def check(backend: str | None = None, group=None) -> None:
    """Raise if an in-kernel collective wait gave up (peer missing / too slow)."""
    c = _comms.get((backend, id(group)))
    if c is not None and hasattr(c, "check"):
        c.check()


def close_all() -> None:
    for c in _comms.values():
        if hasattr(c, "close"):
            c.close()
    _comms.clear()


def ring_allreduce_simulate(ranks: list[torch.Tensor]) -> list[torch.Tensor]:
    """The reference's in-process ring all-reduce over a list of per-rank tensors (sum)."""
    p = len(ranks)
    n = ranks[0].numel()
    chunk = -(-n // p)
    bufs = []
    for t in ranks:
        b = torch.zeros(p * chunk, dtype=t.dtype)
        b[:n] = t.reshape(-1)
        bufs.append(b.view(p, chunk))
    for step in range(p - 1):  # reduce-scatter
        sends = [bufs[r][(r - step) % p].clone() for r in range(p)]
        for r in range(p):
            bufs[(r + 1) % p][(r - step) % p] += sends[r]
    for step in range(p - 1):  # all-gather
        sends = [bufs[r][(r + 1 - step) % p].clone() for r in range(p)]
        for r in range(p):
            bufs[(r + 1) % p][(r + 1 - step) % p] = sends[r]
    return [b.view(-1)[:n].view_as(t) for b, t in zip(bufs, ranks)]


class RingTopology:
    def __init__(self, world_size: int):
        self.world = world_size

    def left_neighbor(self, rank: int) -> int:
        return (rank - 1) % self.world

    def right_neighbor(self, rank: int) -> int:
        return (rank + 1) % self.world


class TreeTopology:
    def __init__(self, world_size: int):
        self.world = world_size

    def parent(self, rank: int) -> int | None:
        return None if rank == 0 else (rank - 1) // 2

    def children(self, rank: int) -> list[int]:
        return [c for c in (2 * rank + 1, 2 * rank + 2) if c < self.world]


def split_tensor_for_allreduce(t: torch.Tensor, parts: int) -> list[torch.Tensor]:
    return list(torch.tensor_split(t.reshape(-1), parts))


def concat_chunks(chunks: list[torch.Tensor]) -> torch.Tensor:
    return torch.cat([c.reshape(-1) for c in chunks])


def shard_tensor_for_rank(t: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    return torch.tensor_split(t, world, dim=dim)[rank].contiguous()


class Work:
    """Handle of a collective started with ``*_async`` (reference ``AsyncCollective::wait``,
    crates/brain-distributed/src/async_exec.rs:6-18). On CUDA the collective runs on a side stream
    and ``wait()`` makes the caller's current stream wait for it (no host block); on CPU it wraps the
    process-group work object."""

    def __init__(self, result, event=None, work=None):
        self.result, self._event, self._work = result, event, work

    def wait(self):
        if self._work is not None:
            self._work.wait()
        elif self._event is not None:
            torch.cuda.current_stream().wait_event(self._event)
        return self.result

    def is_completed(self) -> bool:
        if self._work is not None:
            return self._work.is_completed()
        return self._event is None or self._event.query()


_side_streams: dict = {}


def _run_async(fn, t: torch.Tensor, *args, **kw) -> Work:
    if _world(kw.get("group")) == 1:
        return Work(t)
    if not t.is_cuda:
        if fn is all_reduce and kw.get("op", "sum") == "sum":
            return Work(t, work=dist.all_reduce(t, group=kw.get("group"), async_op=True))
        return Work(fn(t, *args, **kw))
    s = _side_streams.get(t.device)
    if s is None:
        s = _side_streams[t.device] = torch.cuda.Stream(t.device)
    s.wait_stream(torch.cuda.current_stream(t.device))
    with torch.cuda.stream(s):
        out = fn(t, *args, **kw)
        ev = torch.cuda.Event()
        ev.record(s)
    t.record_stream(s)
    return Work(out, event=ev)


def all_reduce_async(t: torch.Tensor, op: str = "sum", group=None, backend: str | None = None) -> Work:
    return _run_async(all_reduce, t, op=op, group=group, backend=backend)


def all_gather_async(t: torch.Tensor, group=None, backend: str | None = None) -> Work:
    return _run_async(all_gather, t, group=group, backend=backend)


def reduce_scatter_async(t: torch.Tensor, group=None, backend: str | None = None, op: str = "sum") -> Work:
    return _run_async(reduce_scatter, t, group=group, backend=backend, op=op)
