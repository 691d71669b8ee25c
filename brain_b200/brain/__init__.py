"""The reference's Python package API (``import brain``), on this framework.

Reference: python/brain/__init__.py (``Tensor, Value, zeros, ones, tensor, nn, optim``) over the pyo3
module of crates/brain-python/src (``PyTensor`` tensor.rs, ``PyValue`` autograd.rs, ``PyLinear`` /
``PyConv2d`` / ``PyLayerNorm`` / ``PyMSELoss`` / ``PyCrossEntropyLoss`` nn.rs, ``PyAdam`` / ``PyAdamW`` /
``PySgd`` optim.rs) and its contract in tests/python/test_{tensor,autograd,nn,optim,integration}.py:
shapes are Python lists, ``numel`` is a property, ``to_list()`` flattens row-major, ``item()`` raises
``ValueError`` unless the tensor has one element, a ``Value``'s ``grad`` is ``None`` until backward and
is reset to ``None`` by ``zero_grad``, ``backward()`` on a non-scalar seeds ones, and ``nn.Module``
finds the Values, Tensors and sub-modules stored on it.

Usage: ``import brain_b200.brain as brain``. Data are float32 torch tensors (the reference computes in
f64); ``to(device)`` moves them to a GPU, where ``Linear`` on bf16 inputs runs the tcgen05 GEMM.
"""
from __future__ import annotations

import torch

from . import nn, optim  # noqa: F401
from ._core import Tensor, Value, ones, tensor, zeros  # noqa: F401

__all__ = ["Tensor", "Value", "zeros", "ones", "tensor", "nn", "optim"]
