"""Process-group bootstrap and rank context (one process per GPU).

``init()`` reads RANK / LOCAL_RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT (torchrun conventions),
binds the process to its GPU and creates the default process group (NCCL on GPUs, Gloo on CPU)
with a bounded timeout so that ranks waiting on a dead peer fail instead of hanging.

Reference: ``DistributedContext{rank, world_size, local_rank}``, ``is_master``
(crates/brain-distributed/src/core.rs:13-33), ``ProcessGroup{name, ranks}`` (group.rs:7-25),
``DistributedConfig.timeout_ms = 30000`` (config.rs:19-28), rank log prefix ``[Rank r/W]`` (helper.rs:8).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist


@dataclass
class DistributedContext:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    backend: str = "none"
    device: torch.device = field(default_factory=lambda: torch.device("cpu"))

    @property
    def is_master(self) -> bool:
        return self.rank == 0

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1


@dataclass
class ProcessGroup:
    name: str
    ranks: list[int]
    handle: object = None

    def size(self) -> int:
        return len(self.ranks)


_CTX: DistributedContext | None = None


def env_world() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", os.environ.get("RANK", "0"))))


def init(backend: str | None = None, timeout_s: float = 120.0, device: str | None = None) -> DistributedContext:
    """Initialise (idempotent) and return the rank context."""
    global _CTX
    if _CTX is not None:
        return _CTX
    rank, world, local = env_world()
    use_cuda = torch.cuda.is_available() and device != "cpu"
    if use_cuda:
        torch.cuda.set_device(local % torch.cuda.device_count())
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = torch.device("cpu")
    be = "none"
    if world > 1:
        be = backend or ("nccl" if use_cuda else "gloo")
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29500")
        if not dist.is_initialized():
            kw = dict(backend=be, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
            if be == "nccl":
                kw["device_id"] = dev
            dist.init_process_group(**kw)
    _CTX = DistributedContext(rank, world, local, be, dev)
    return _CTX


def context() -> DistributedContext:
    return _CTX if _CTX is not None else DistributedContext(*env_world()[:2], env_world()[2])


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def shutdown() -> None:
    global _CTX
    if dist.is_initialized():
        dist.destroy_process_group()
    _CTX = None


def rank_prefix(rank: int | None = None, world: int | None = None) -> str:
    c = context()
    return f"[Rank {c.rank if rank is None else rank}/{c.world_size if world is None else world}]"


def new_group(ranks: list[int], name: str = "group") -> ProcessGroup:
    h = dist.new_group(ranks) if dist.is_initialized() else None
    return ProcessGroup(name, list(ranks), h)


@dataclass
class ParallelMesh:
    """Rank layout (pp, dp, tp) with tensor-parallel ranks adjacent (the fastest-varying coordinate, so
    a TP group sits on neighbouring GPUs of one NVSwitch domain), then data-parallel, then pipeline.
    ``tp_group`` / ``dp_group`` / ``pp_group`` are this rank's subgroups."""
    tp: int
    dp: int
    pp: int
    rank: int
    tp_rank: int
    dp_rank: int
    pp_rank: int
    tp_group: ProcessGroup
    dp_group: ProcessGroup
    pp_group: ProcessGroup

    @staticmethod
    def coords(rank: int, tp: int, dp: int) -> tuple[int, int, int]:
        return rank // (tp * dp), (rank // tp) % dp, rank % tp


def init_mesh(tp: int = 1, pp: int = 1) -> ParallelMesh:
    """Collective: builds every TP, DP and PP subgroup (every rank creates all of them, in the same
    order, as ``torch.distributed.new_group`` requires) and returns this rank's view."""
    c = context()
    W = c.world_size
    if W % (tp * pp):
        raise ValueError(f"world size {W} is not divisible by tp {tp} x pp {pp}")
    dp = W // (tp * pp)
    pr, dr, tr = ParallelMesh.coords(c.rank, tp, dp)
    mine = {}
    for p in range(pp):
        for d in range(dp):
            ranks = [p * tp * dp + d * tp + t for t in range(tp)]
            g = new_group(ranks, f"tp{p}.{d}")
            if c.rank in ranks:
                mine["tp"] = g
    for p in range(pp):
        for t in range(tp):
            ranks = [p * tp * dp + d * tp + t for d in range(dp)]
            g = new_group(ranks, f"dp{p}.{t}")
            if c.rank in ranks:
                mine["dp"] = g
    for d in range(dp):
        for t in range(tp):
            ranks = [p * tp * dp + d * tp + t for p in range(pp)]
            g = new_group(ranks, f"pp{d}.{t}")
            if c.rank in ranks:
                mine["pp"] = g
    return ParallelMesh(tp, dp, pp, c.rank, tr, dr, pr, mine["tp"], mine["dp"], mine["pp"])
