"""Communication backends behind the public collectives and the data-parallel engine.

``NcclComm`` issues NCCL collectives through ``torch.distributed`` (Gloo on CPU ranks): it is the
reference / baseline path and the fallback. The in-kernel NVLink backend lives in
``parallel.symm`` and exposes the same methods plus the fused ones.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class NcclComm:
    name = "nccl"
    fused_rs_adamw = None

    def __init__(self, group=None):
        self.group = group

    @property
    def world_size(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    @property
    def rank(self) -> int:
        return dist.get_rank(self.group) if dist.is_initialized() else 0

    def all_reduce(self, t: torch.Tensor, op: str = "sum") -> torch.Tensor:
        if self.world_size > 1:
            dist.all_reduce(t, op=_op(op), group=self.group)
        return t

    def reduce_scatter_flat(self, full: torch.Tensor, out: torch.Tensor, op: str = "sum") -> torch.Tensor:
        if self.world_size > 1:
            dist.reduce_scatter_tensor(out, full, op=_op(op), group=self.group)
        else:
            out.copy_(full)
        return out

    def all_gather_flat(self, shard: torch.Tensor, full: torch.Tensor) -> torch.Tensor:
        if self.world_size > 1:
            dist.all_gather_into_tensor(full, shard, group=self.group)
        else:
            full.copy_(shard)
        return full

    def broadcast(self, t: torch.Tensor, src: int = 0) -> torch.Tensor:
        if self.world_size > 1:
            dist.broadcast(t, src, group=self.group)
        return t


def _op(op: str):
    return {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN,
            "avg": dist.ReduceOp.AVG, "mean": dist.ReduceOp.AVG, "prod": dist.ReduceOp.PRODUCT}[op]
