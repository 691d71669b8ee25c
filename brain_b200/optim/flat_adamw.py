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
    def step(self, grad_scale: float = 1.0, check_finite: bool = False) -> None:
        world = self.flat.world_size
        self.flat.absorb_grads()
        self.step_count += 1
        b1, b2 = self.betas
        if (world > 1 and self.comm is not None and getattr(self.comm, "fused_rs_adamw", None) is not None
                and not check_finite and self.vmax is None):
            # one kernel: NVLink reduce-scatter + un-scale + AdamW + bf16 weights pushed to every rank
            self.comm.fused_rs_adamw(self, grad_scale / world)
            return
        else:
            if world > 1:
                self.comm.reduce_scatter_flat(self.flat.grad_buf, self.grad_shard())
                scale = grad_scale / world
            else:
                scale = grad_scale
            g = self.grad_shard()
            fi = None
            if check_finite:
                self.found_inf.zero_()
                K.sumsq(g, scale, found_inf=self.found_inf)
                fi = self.found_inf
            K.adamw_(self.master, self.m, self.v, g, lr=self.lr, beta1=b1, beta2=b2, eps=self.eps,
                     weight_decay=self.weight_decay, step=self.step_count, grad_scale=scale,
                     p16=self.flat.shard(self.flat.param_buf), vmax=self.vmax, found_inf=fi)
        if world > 1:
            self.comm.all_gather_flat(self.flat.shard(self.flat.param_buf), self.flat.param_buf)

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
