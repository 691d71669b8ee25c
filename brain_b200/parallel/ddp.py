"""Data-parallel training engine (``brain_b200.parallel.DataParallel``).

Replicates the model on every rank, reduces gradients by the **mean** (the reference's reduction,
crates/brain-distributed/src/data_parallel.rs:48-63) and shards the AdamW state across ranks:
  * parameters live in one flat bf16 buffer and gradients in one flat ``main_grad`` buffer
    (``parallel.flat``), written in place by the backward kernels;
  * the optimizer step is a reduce-scatter of the gradient bucket, the fused AdamW over the local
    shard and an all-gather of the updated bf16 shards (``optim.flat_adamw``);
  * with the NVLink backend (``comm="nvlink"``) the reduce-scatter, un-scaling and AdamW update run
    as one kernel that pulls peers' gradient shards over NVLink (``parallel.symm``); with
    ``overlap=True`` that kernel runs per bucket of blocks during backward (``parallel.overlap``).

The reference's helpers are kept: ``sync_gradients`` (scale by 1/world after a sum) and
``sync_ensemble_gradients`` (average per-parameter gradients of in-process "ranks").
"""
from __future__ import annotations

import torch

from ..optim.flat_adamw import FlatAdamW
from . import dist as _dist
from .comm import NcclComm
from .flat import FlatParams


class DataParallel:
    def __init__(self, model: torch.nn.Module, lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.0, grad_dtype: torch.dtype = torch.float32, comm: str | object = "nccl",
                 loss_fn=None, overlap: bool = False, bucket_bytes: int = 512 << 20, overlap_mode: str = "ce",
                 grad_scaler=None, max_grad_norm: float = 0.0, check_finite: bool = False):
        """``grad_scaler`` (``autograd.GradScaler``): dynamic loss scaling; the loss is multiplied by the
        scaler's scale, the gradient divided by it inside the optimizer kernel, and a step with any
        non-finite gradient element on any rank is skipped on every rank before the scale backs off.
        ``max_grad_norm``: clip by the global norm over all ranks. ``check_finite``: skip non-finite
        steps without loss scaling. The three make the step guarded: gradient statistics are reduced
        over the ranks on the device before AdamW, and the host reads the skip flag once per step."""
        ctx = _dist.context()
        self.ctx = ctx
        self.model = model
        if isinstance(comm, str):
            if comm == "nvlink" and ctx.world_size > 1:
                from .symm import NvlinkComm
                comm = NvlinkComm()
            else:
                comm = NcclComm()
        self.comm = comm
        alloc = comm.alloc if getattr(comm, "name", "") == "nvlink" else None
        self.flat = FlatParams(list(model.parameters()), ctx.world_size, ctx.rank, grad_dtype, alloc=alloc)
        if ctx.world_size > 1:
            self.comm.broadcast(self.flat.param_buf, 0)
        self.optimizer = FlatAdamW(self.flat, lr, betas, eps, weight_decay, comm=self.comm)
        self.loss_fn = loss_fn
        self.grad_scaler = grad_scaler
        self.max_grad_norm = float(max_grad_norm)
        self.check_finite = check_finite
        self.after_backward: list = []  # callables fn(dp) run after backward, before the reduction finishes
        self.skipped_steps = 0
        self.steps = 0
        self.overlapped = None
        if overlap and self.flat.grad_buf.is_cuda and (ctx.world_size == 1 or
                                                         getattr(self.comm, "name", "") == "nvlink"):
            from .overlap import OverlappedStep
            self.overlapped = OverlappedStep(self, bucket_bytes=bucket_bytes, mode=overlap_mode)

    @property
    def world_size(self) -> int:
        return self.ctx.world_size

    @property
    def rank(self) -> int:
        return self.ctx.rank

    def forward_loss(self, *batch):
        if self.loss_fn is not None:
            return self.loss_fn(self.model, *batch)
        return self.model.loss(*batch)

    def guarded(self) -> bool:
        return (self.grad_scaler is not None and self.grad_scaler.enabled) or self.max_grad_norm > 0 or \
            self.check_finite

    def train_step(self, *batch, loss_scale: float = 1.0) -> torch.Tensor:
        """zero grads -> forward -> backward -> reduce-scatter + sharded AdamW -> all-gather.

        Returns the local loss (device scalar, not synchronised; with a guarded step the host has
        read the skip flag, so the step is complete).
        """
        scaler = self.grad_scaler if (self.grad_scaler is not None and self.grad_scaler.enabled) else None
        if scaler is not None:
            loss_scale = scaler.scale
        guarded = self.guarded()
        self.optimizer.zero_grad()
        if self.overlapped is not None:
            # reduction + AdamW of each bucket start during backward (parallel.overlap)
            self.overlapped.arm(1.0 / loss_scale / self.world_size, guarded=guarded, max_norm=self.max_grad_norm)
        loss = self.forward_loss(*batch)
        (loss * loss_scale if loss_scale != 1.0 else loss).backward()
        if self.after_backward:
            if self.overlapped is None:
                self.flat.absorb_grads()  # hooks see the complete flat gradient
            for fn in self.after_backward:
                fn(self)
        if self.overlapped is not None:
            self.overlapped.finish()
        else:
            self.optimizer.step(grad_scale=1.0 / loss_scale, check_finite=guarded, max_norm=self.max_grad_norm)
        if guarded:
            skipped = self.optimizer.undo_skipped()
            self.skipped_steps += int(skipped)
            if scaler is not None:
                scaler.update(skipped)
        self.steps += 1
        return loss.detach()

    def grad_norm(self) -> float:
        """Global gradient norm of the last guarded step (before clipping), over all ranks."""
        return self.optimizer.grad_norm()

    def save_checkpoint(self, directory: str, metadata: dict | None = None) -> None:
        """Collective: every rank writes its optimizer-state shard, rank 0 the weights
        (``checkpoint.sharded``)."""
        from ..checkpoint.sharded import save_sharded
        save_sharded(self, directory, metadata)

    def load_checkpoint(self, directory: str) -> dict:
        """Collective: restores weights and this rank's optimizer state, from any saved world size."""
        from ..checkpoint.sharded import load_sharded
        meta = load_sharded(self, directory)
        self.steps = self.optimizer.step_count
        return meta

    def sync_gradients(self) -> None:
        """All-reduce gradients as the mean over ranks (flat bucket, in place)."""
        self.flat.absorb_grads()
        if self.world_size > 1:
            self.comm.all_reduce(self.flat.grad_buf)
            self.flat.grad_buf.mul_(1.0 / self.world_size)

    @staticmethod
    def sync_ensemble_gradients(rank_grads: list[list[torch.Tensor]]) -> None:
        """Average gradients of in-process replicas in place (reference behaviour, for tests)."""
        n = len(rank_grads)
        for i in range(len(rank_grads[0])):
            mean = sum(r[i] for r in rank_grads) / n
            for r in rank_grads:
                r[i].copy_(mean)
