"""Module system with the reference's API names, built on ``torch.nn.Module``.

Reference: the brain-nn ``Module`` trait (``forward``, ``parameters``, ``set_training``,
``state_dict``/``load_state_dict``; crates/brain-nn/src/module/mod.rs:50-165) and its containers
``Sequential``/``ModuleList``/``ModuleDict`` (crates/brain-nn/src/containers/seq.rs:9). PyTorch's
module machinery provides parameter registration, device movement and hooks (the reference's
``HookRegistry``, crates/brain-nn/src/hooks.rs:16, maps to forward (pre-)hooks).
"""
from __future__ import annotations

import torch


class Module(torch.nn.Module):
    """Base module. Adds the reference's helper names on top of ``torch.nn.Module``."""

    def set_training(self, mode: bool = True) -> "Module":
        return self.train(mode)

    def is_training(self) -> bool:
        return self.training

    def num_parameters(self, trainable_only: bool = False) -> int:
        return sum(p.numel() for p in self.parameters() if p.requires_grad or not trainable_only)

    def named_parameter_list(self):
        return list(self.named_parameters())

    def forward_tensor(self, x: torch.Tensor) -> torch.Tensor:
        """Inference forward without gradient tracking (reference ``forward_tensor`` shim)."""
        with torch.no_grad():
            return self.forward(x)

    def zero_grad(self, set_to_none: bool = True) -> None:  # keeps flat main_grad buffers intact
        super().zero_grad(set_to_none=set_to_none)


class Sequential(torch.nn.Sequential, Module):
    pass


class ModuleList(torch.nn.ModuleList, Module):
    pass


class ModuleDict(torch.nn.ModuleDict, Module):
    pass


class Identity(Module):
    def forward(self, x):
        return x
