"""Optimizers (fused AdamW / SGD kernels over flat buffers, plus the reference's optimizer family)."""
from .flat_adamw import FlatAdamW  # noqa: F401
