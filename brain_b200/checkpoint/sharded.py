"""Sharded training checkpoints for the data-parallel engine: every rank writes its own piece of the
float32 optimizer state (master weights, first and second moments), rank 0 writes the bf16 model
weights by name, and loading re-shards the state onto any world size.

Reference: optimizer state in checkpoints (crates/brain-optim/src/adam/mod.rs:251-283 ``adam_m_{i}`` /
``adam_v_{i}``, OptimizerCheckpoint state.rs:174) and Trainer resume (crates/brain-train/tests/
trainer_regression.rs:99-142). The reference keeps the whole state in one process; here the state is
sharded (ZeRO-1), so a checkpoint is one file per rank plus the model file, all in the native-dtype
BRAINCK2 container (per-tensor CRC32, sorted, deterministic).

Each rank owns a list of pieces (global offset, length) of the flat parameter buffer: one contiguous
shard for the flat optimizer, or one piece per bucket for the overlapped reduction. A rank file stores
its pieces and the concatenated state; loading assembles the full flat vectors from every file and
cuts out the new rank's pieces. Parameter offsets in the flat buffer do not depend on the world size
(only the padding at the end does), so any old and new world sizes combine.
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

from .formats import CheckpointError, load_brain_v2, save_brain_v2


def _layout(dp):
    """(pieces [(global offset, length, state offset)], master, exp_avg, exp_avg_sq) of this rank."""
    ov = getattr(dp, "overlapped", None)
    if ov is not None:
        return list(ov.pieces), ov.master, ov.m, ov.v
    f, o = dp.flat, dp.optimizer
    return [(f.rank * f.shard_size, f.shard_size, 0)], o.master, o.m, o.v


def _barrier():
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def rank_file(directory: str, rank: int) -> str:
    return os.path.join(directory, f"optim-rank{rank:05d}.brain2")


def save_sharded(dp, directory: str, metadata: dict | None = None) -> None:
    """Collective: every rank of ``dp`` must call it."""
    os.makedirs(directory, exist_ok=True)
    f, opt = dp.flat, dp.optimizer
    pieces, master, m, v = _layout(dp)
    tensors = {"pieces": torch.tensor([[a, n, s] for a, n, s in pieces], dtype=torch.int64).reshape(-1, 3),
               "master": master.detach().cpu(), "exp_avg": m.detach().cpu(), "exp_avg_sq": v.detach().cpu()}
    meta = {"rank": f.rank, "world_size": f.world_size, "step": opt.step_count, "lr": opt.lr,
            "betas": list(opt.betas), "eps": opt.eps, "weight_decay": opt.weight_decay, "numel": f.numel,
            "padded": f.padded}
    save_brain_v2(rank_file(directory, f.rank), tensors, meta)
    if f.rank == 0:
        named = {n: p.detach().cpu() for n, p in dp.model.named_parameters() if p.requires_grad}
        save_brain_v2(os.path.join(directory, "model.brain2"), named, dict(metadata or {}))
        with open(os.path.join(directory, "index.json"), "w") as fh:
            json.dump({"format": "brain-sharded-1", "world_size": f.world_size, "step": opt.step_count,
                       "numel": f.numel, "files": [os.path.basename(rank_file(directory, r))
                                                   for r in range(f.world_size)]}, fh, sort_keys=True)
    _barrier()


def load_full_state(directory: str) -> tuple[dict, dict]:
    """Assembles the full flat master / exp_avg / exp_avg_sq vectors from every rank file."""
    with open(os.path.join(directory, "index.json")) as fh:
        index = json.load(fh)
    full, meta0 = None, None
    for name in index["files"]:
        t, meta = load_brain_v2(os.path.join(directory, name))
        if meta0 is None:
            meta0 = meta
            n = int(meta["padded"])
            full = {k: torch.zeros(n, dtype=torch.float32) for k in ("master", "exp_avg", "exp_avg_sq")}
        elif int(meta["step"]) != int(meta0["step"]):
            raise CheckpointError(f"{name}: step {meta['step']} differs from rank 0's {meta0['step']}")
        for a, n, s in t["pieces"].tolist():
            for k in full:
                full[k][a:a + n] = t[k][s:s + n]
    return full, meta0


def load_sharded(dp, directory: str) -> dict:
    """Restores weights and this rank's optimizer state (any saved world size). Returns the model file's
    metadata."""
    full, meta = load_full_state(directory)
    named, model_meta = load_brain_v2(os.path.join(directory, "model.brain2"))
    params = dict(dp.model.named_parameters())
    missing = [n for n in named if n not in params]
    if missing:
        raise CheckpointError(f"checkpoint has parameters the model lacks: {missing[:5]}")
    f, opt = dp.flat, dp.optimizer
    if int(meta["numel"]) != f.numel:
        raise CheckpointError(f"flat size {meta['numel']} in the checkpoint, {f.numel} in the model")
    with torch.no_grad():
        for n, t in named.items():
            params[n].copy_(t.to(params[n].device, params[n].dtype))
        pieces, master, m, v = _layout(dp)
        for a, n, s in pieces:
            hi = min(a + n, full["master"].numel())
            k = max(0, hi - a)
            for dst, key in ((master, "master"), (m, "exp_avg"), (v, "exp_avg_sq")):
                dst[s:s + n].zero_()
                if k:
                    dst[s:s + k].copy_(full[key][a:a + k].to(dst.device))
    opt.step_count = int(meta["step"])
    opt.lr = float(meta["lr"])
    opt.betas = tuple(meta["betas"])
    opt.eps = float(meta["eps"])
    opt.weight_decay = float(meta["weight_decay"])
    _barrier()
    return model_meta
