"""Weight pruning: magnitude masks, structured (row) masks, global pruning of a module, and masks kept
in force through a forward pre-hook.

Reference: crates/brain-nn/src/pruning.rs:10-50 (``PruningMask::from_magnitude(weight, sparsity)``,
``apply``) and the hook registry (crates/brain-nn/src/hooks.rs:16), here ``torch.nn.Module`` forward
pre-hooks.
"""
from __future__ import annotations

import torch


class PruningMask:
    def __init__(self, mask: torch.Tensor):
        self.mask = mask.bool()

    @classmethod
    def from_magnitude(cls, weight: torch.Tensor, sparsity: float) -> "PruningMask":
        """Zeroes the ``round(sparsity * n)`` smallest-magnitude entries (ties broken by position)."""
        n = weight.numel()
        k = int(round(min(max(sparsity, 0.0), 1.0) * n))
        mask = torch.ones(n, dtype=torch.bool, device=weight.device)
        if k:
            idx = torch.argsort(weight.detach().abs().reshape(-1).float(), stable=True)[:k]
            mask[idx] = False
        return cls(mask.view_as(weight))

    @classmethod
    def structured_rows(cls, weight: torch.Tensor, sparsity: float) -> "PruningMask":
        """Removes whole output rows with the smallest L2 norms."""
        rows = weight.shape[0]
        k = int(round(min(max(sparsity, 0.0), 1.0) * rows))
        mask = torch.ones_like(weight, dtype=torch.bool)
        if k:
            norms = weight.detach().float().reshape(rows, -1).norm(dim=1)
            mask[torch.argsort(norms, stable=True)[:k]] = False
        return cls(mask)

    def apply(self, weight: torch.Tensor) -> torch.Tensor:
        return weight * self.mask.to(weight.dtype)

    def sparsity(self) -> float:
        return 1.0 - float(self.mask.float().mean())


def prune_module(module: torch.nn.Module, sparsity: float, structured: bool = False, global_: bool = False,
                 param_filter=lambda name, p: p.dim() >= 2) -> dict:
    """Masks every selected weight (``global_``: one threshold over all of them), zeroes the pruned
    entries in place, and registers a forward pre-hook that re-applies the masks (so optimizer steps
    cannot revive them). Returns {parameter name: PruningMask}."""
    params = [(n, p) for n, p in module.named_parameters() if param_filter(n, p)]
    masks = {}
    if global_ and not structured:
        allw = torch.cat([p.detach().abs().reshape(-1).float() for _, p in params])
        k = int(round(sparsity * allw.numel()))
        thr = torch.kthvalue(allw.cpu(), k).values.item() if k else -1.0
        for n, p in params:
            masks[n] = PruningMask(p.detach().abs().float() > thr)
    else:
        for n, p in params:
            masks[n] = (PruningMask.structured_rows if structured else PruningMask.from_magnitude)(p, sparsity)
    lookup = dict(module.named_parameters())

    def reapply(mod, args):
        with torch.no_grad():
            for n, m in masks.items():
                lookup[n].mul_(m.mask.to(lookup[n].dtype))

    reapply(module, ())
    module._brain_pruning_hook = module.register_forward_pre_hook(reapply)
    return masks


def remove_pruning(module: torch.nn.Module) -> None:
    h = getattr(module, "_brain_pruning_hook", None)
    if h is not None:
        h.remove()
        del module._brain_pruning_hook
