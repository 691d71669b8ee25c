"""Sharded AdamW over flat buffers (ZeRO-1): the optimizer of the data-parallel engine.

Each rank keeps float32 master weights and both moments for its shard only. A step is
    1. gradient reduce-scatter over the flat bucket (sum; the 1/world mean and 1/loss-scale are
       folded into ``grad_scale``),
    2. one fused AdamW kernel over the shard (reference order, crates/brain-optim/src/adam/mod.rs:128-200)
       that also writes the bf16 compute weights of the shard,
    3. a parameter all-gather of the bf16 shards.
With one rank steps 1 and 3 vanish and the kernel runs over the whole model.

The collectives go through a ``comm`` object (``parallel.comm``): the NCCL backend for the
reference path or the in-kernel NVLink backend whose reduce-scatter is fused with the AdamW update.
"""
from __future__ import annotations

import torch

from ..ops import optim_kernels as K


class FlatAdamW:
    def __init__(self, flat, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, amsgrad: bool = False, comm=None):
        self.flat = flat
        self.lr, self.betas, self.eps, self.weight_decay, self.amsgrad = lr, betas, eps, weight_decay, amsgrad
        self.comm = comm
        shard = flat.shard(flat.param_buf)
        self.master = shard.float().clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.vmax = torch.zeros_like(self.master) if amsgrad else None
        self.step_count = 0
        self.found_inf = torch.zeros(1, device=shard.device, dtype=torch.int32)
        self.stats = torch.zeros(2, device=shard.device, dtype=torch.float32)  # (sum of squares, non-finite)
        self.coef = torch.ones(1, device=shard.device, dtype=torch.float32)
        self._guarded = False

    @property
    def param_groups(self):
        return [{"lr": self.lr, "betas": self.betas, "eps": self.eps, "weight_decay": self.weight_decay}]

    def set_lr(self, lr: float) -> None:
        self.lr = lr

    def get_lr(self) -> float:
        return self.lr

    def zero_grad(self) -> None:
        self.flat.zero_grad()

    def grad_shard(self) -> torch.Tensor:
        return self.flat.shard(self.flat.grad_buf)

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, check_finite: bool = False, max_norm: float = 0.0) -> None:
        """One sharded AdamW step on the flat gradient bucket.

        ``grad_scale`` multiplies the summed gradient (1/world and 1/loss-scale are folded in here).
        With ``check_finite`` or ``max_norm > 0`` the step is guarded: the reduced gradient's sum of
        squares and a non-finite flag are reduced over all ranks on the device, every rank skips the
        step alike when any element anywhere is non-finite (``found_inf`` is set; dynamic loss scaling,
        crates/brain-autograd/src/engine/mixed.rs:49-95), and the gradient is scaled by the global-norm
        clip coefficient min(1, max_norm / (norm + 1e-6)) (crates/brain-optim/src/clipping/norm.rs:38).
        ``grad_norm()`` then returns the global norm of the un-clipped gradient."""
        world = self.flat.world_size
        self.flat.absorb_grads()
        self.step_count += 1
        b1, b2 = self.betas
        guarded = check_finite or max_norm > 0
        fused = world > 1 and self.comm is not None and getattr(self.comm, "fused_rs_adamw", None) is not None
        if fused and not guarded and self.vmax is None:
            # one kernel: NVLink reduce-scatter + un-scale + AdamW + bf16 weights pushed to every rank
            self.comm.fused_rs_adamw(self, grad_scale / world)
            return
        g = self.grad_shard()
        scale = grad_scale / world if world > 1 else grad_scale
        if world > 1:
            if guarded and fused:
                # NVLink: sum the peers' pieces of this rank's shard into the local shard, scaled
                self.comm.reduce_scatter_inplace(self.flat.grad_buf, g, scale)
                scale = 1.0
            else:
                self.comm.reduce_scatter_flat(self.flat.grad_buf, g)
        fi = coef = None
        if guarded:
            K.grad_stats(g, scale, self.stats)
            if world > 1:
                self.comm.all_reduce(self.stats)
            fi, coef = K.step_guard(self.stats, max_norm, self.found_inf, self.coef)
        K.adamw_(self.master, self.m, self.v, g, lr=self.lr, beta1=b1, beta2=b2, eps=self.eps,
                 weight_decay=self.weight_decay, step=self.step_count, grad_scale=scale,
                 p16=self.flat.shard(self.flat.param_buf), vmax=self.vmax, found_inf=fi, coef=coef)
        if guarded:
            # a skipped step does not count towards the bias corrections (the host learns it when the
            # caller reads found_inf; ``undo_skipped`` rolls the counter back)
            self._guarded = True
        if world > 1:
            self.comm.all_gather_flat(self.flat.shard(self.flat.param_buf), self.flat.param_buf)

    def skipped(self) -> bool:
        """Whether the last guarded step was skipped (reads the device flag: synchronises)."""
        return bool(int(self.found_inf.item()))

    def undo_skipped(self) -> bool:
        """After a guarded step: if it was skipped, roll the step counter back; returns the flag."""
        bad = self.skipped()
        if bad:
            self.step_count -= 1
        return bad

    def grad_norm(self) -> float:
        """Global L2 norm of the gradient of the last guarded step (before clipping)."""
        return float(self.stats[0].clamp_min(0).sqrt())

    def state_dict(self) -> dict:
        return {"step": self.step_count, "lr": self.lr, "betas": self.betas, "eps": self.eps,
                "weight_decay": self.weight_decay, "master": self.master, "exp_avg": self.m, "exp_avg_sq": self.v,
                "rank": self.flat.rank, "world_size": self.flat.world_size}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        self.lr = float(sd["lr"])
        self.master.copy_(sd["master"])
        self.m.copy_(sd["exp_avg"])
        self.v.copy_(sd["exp_avg_sq"])
        self.flat.shard(self.flat.param_buf).copy_(self.master)
