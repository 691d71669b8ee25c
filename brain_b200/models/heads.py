"""Output heads and the transformer embedding layer.

Reference: crates/brain-transformer/src/head/mod.rs:19-130 (``LmHead`` with an optional tied weight,
``ClsHead`` pooling the first token through a tanh dense layer before the classifier) and
src/embedding_layers.rs:22-200 (``TransformerEmbedding``: token embedding plus optional learned
positions and token types, then an optional LayerNorm / RMSNorm).

The projections go through ``brain_b200.nn.Linear`` / ``ops.linear`` (the tcgen05 GEMM for bf16 CUDA
tensors), the embedding gather through ``ops.embedding`` and the norms through the norm kernels.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from ..nn.layers import Embedding, LayerNorm, Linear, RMSNorm
from ..nn.module import Module


@dataclass
class HeadConfig:
    hidden_dim: int
    vocab_size: int = 0
    num_labels: int = 2
    bias: bool = False


class LmHead(Module):
    """hidden [.., d] -> logits [.., vocab]; ``tied`` reuses an embedding matrix [vocab, d]."""

    def __init__(self, config: HeadConfig, tied: torch.Tensor | None = None, device=None, dtype=None):
        super().__init__()
        self.config = config
        self.tied = tied
        self.proj = None if tied is not None else Linear(config.hidden_dim, config.vocab_size, config.bias, device, dtype)

    @classmethod
    def new_tied(cls, config: HeadConfig, embedding_weight: torch.Tensor) -> "LmHead":
        return cls(config, tied=embedding_weight)

    def forward(self, h):
        return ops.linear(h, self.tied) if self.tied is not None else self.proj(h)


class ClsHead(Module):
    """First-token pooling: tanh(W_p h[:, 0] + b_p), then the classifier."""

    def __init__(self, config: HeadConfig, device=None, dtype=None):
        super().__init__()
        self.pool = Linear(config.hidden_dim, config.hidden_dim, True, device, dtype)
        self.cls = Linear(config.hidden_dim, config.num_labels, True, device, dtype)

    def forward(self, h):
        return self.cls(torch.tanh(self.pool(h[:, 0])))


@dataclass
class EmbConfig:
    vocab_size: int
    hidden_dim: int
    max_positions: int = 0      # 0: no learned positions
    type_vocab_size: int = 0    # 0: no token types
    norm: str = "none"          # "none" | "layer" | "rms"
    eps: float = 1e-5


class TransformerEmbedding(Module):
    def __init__(self, config: EmbConfig, device=None, dtype=None):
        super().__init__()
        c = self.config = config
        self.tok = Embedding(c.vocab_size, c.hidden_dim, device, dtype)
        self.pos = Embedding(c.max_positions, c.hidden_dim, device, dtype) if c.max_positions else None
        self.typ = Embedding(c.type_vocab_size, c.hidden_dim, device, dtype) if c.type_vocab_size else None
        with torch.no_grad():
            for e in (self.tok, self.pos, self.typ):
                if e is not None:
                    e.weight.mul_(0.02)
        self.norm = {"layer": lambda: LayerNorm(c.hidden_dim, c.eps, True, device, dtype),
                     "rms": lambda: RMSNorm(c.hidden_dim, c.eps, device, dtype)}.get(c.norm, lambda: None)()

    def forward(self, ids, token_type=None, offset: int = 0):
        h = self.tok(ids)
        if self.pos is not None:
            pos = torch.arange(offset, offset + ids.shape[1], device=ids.device)
            h = h + self.pos(pos)[None]
        if self.typ is not None:
            h = h + self.typ(token_type if token_type is not None else torch.zeros_like(ids))
        return self.norm(h) if self.norm is not None else h
