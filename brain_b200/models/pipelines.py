"""Transformer builder and task pipelines.

Reference: crates/brain-transformer/src/builder.rs:24-140 (``TransformerBuilder``: arch, vocab size,
hidden size, layers, heads, FFN size, activation, norm position / type, position encoding, max length,
``build_config`` with validation) and src/impl.rs:20-100 (``SequenceClassificationPipeline`` over
BertLite with ``predict_class``; ``TextGenerationPipeline`` over GptLite with ``generate``).
``TransformerBuilder.build_model`` also instantiates the matching model family of this framework.
"""
from __future__ import annotations

import dataclasses

import torch

from .config import BertLiteConfig, GptLiteConfig, LlamaLiteConfig, TransformerConfig
from .generate import GenerationConfig


class TransformerBuilder:
    ARCHS = ("llama", "gpt", "bert")

    def __init__(self):
        self._arch = "llama"
        self._cfg = TransformerConfig()

    def arch(self, arch: str) -> "TransformerBuilder":
        if arch not in self.ARCHS:
            raise ValueError(f"unknown architecture '{arch}' (one of {self.ARCHS})")
        self._arch = arch
        presets = {"llama": dict(norm="rms", activation="swiglu", pre_norm=True, causal=True, rope=True,
                                 learned_positions=False, bias=False),
                   "gpt": dict(norm="layer", activation="gelu", pre_norm=True, causal=True, rope=False,
                               learned_positions=True, bias=True),
                   "bert": dict(norm="layer", activation="gelu", pre_norm=False, causal=False, rope=False,
                                learned_positions=True, bias=True)}[arch]
        self._cfg = dataclasses.replace(self._cfg, **presets)
        return self

    def _set(self, **kw) -> "TransformerBuilder":
        self._cfg = dataclasses.replace(self._cfg, **kw)
        return self

    def vocab_size(self, n: int):
        return self._set(vocab_size=n)

    def hidden_dim(self, d: int):
        return self._set(hidden_dim=d)

    def num_layers(self, n: int):
        return self._set(num_layers=n)

    def num_heads(self, n: int):
        return self._set(num_heads=n, num_kv_heads=n)

    def num_kv_heads(self, n: int):
        return self._set(num_kv_heads=n)

    def intermediate_dim(self, d: int):
        return self._set(intermediate_dim=d)

    def activation(self, act: str):
        return self._set(activation=act)

    def norm_position(self, pre: bool):
        return self._set(pre_norm=pre)

    def norm_type(self, kind: str):
        return self._set(norm=kind)

    def pos_encoding(self, kind: str):
        """"rope" | "learned" | "none"."""
        return self._set(rope=kind == "rope", learned_positions=kind == "learned")

    def max_seq_len(self, n: int):
        return self._set(max_seq_len=n)

    def build_config(self) -> TransformerConfig:
        c = self._cfg
        errs = []
        if c.hidden_dim <= 0 or c.num_layers <= 0 or c.num_heads <= 0 or c.vocab_size <= 0:
            errs.append("sizes must be positive")
        elif c.hidden_dim % c.num_heads:
            errs.append(f"hidden_dim {c.hidden_dim} is not divisible by num_heads {c.num_heads}")
        if c.num_kv_heads <= 0 or c.num_heads % c.num_kv_heads:
            errs.append(f"num_heads {c.num_heads} is not a multiple of num_kv_heads {c.num_kv_heads}")
        if c.rope and (c.hidden_dim // max(1, c.num_heads)) % 2:
            errs.append("RoPE needs an even head dimension")
        if errs:
            raise ValueError("; ".join(errs))
        return c

    def build_model(self, device=None, dtype=torch.float32, seed: int = 0):
        c = self.build_config()
        if self._arch == "llama":
            lc = LlamaLiteConfig(c.vocab_size, c.hidden_dim, c.num_layers, c.num_heads, c.num_kv_heads,
                                 c.hidden_dim // c.num_heads, c.intermediate_dim, c.max_seq_len, c.rope_theta, c.norm_eps)
            from .llama import LlamaLite
            return LlamaLite(lc, device=device, dtype=dtype, seed=seed)
        if self._arch == "gpt":
            from .families import GptLite
            return GptLite(GptLiteConfig(c.vocab_size, c.hidden_dim, c.num_layers, c.num_heads, c.intermediate_dim,
                                         c.max_seq_len, c.norm_eps, c.bias), device=device, dtype=dtype, seed=seed)
        from .families import BertLite
        return BertLite(BertLiteConfig(c.vocab_size, c.hidden_dim, c.num_layers, c.num_heads, c.intermediate_dim,
                                       c.max_seq_len, norm_eps=c.norm_eps), device=device, dtype=dtype, seed=seed)


class SequenceClassificationPipeline:
    """BertLite classifier: ids -> class index (argmax of the [CLS] head)."""

    def __init__(self, config: BertLiteConfig, seed: int = 0, device=None, model=None):
        from .families import BertLite
        self.model = model or BertLite(config, device=device, seed=seed)
        self.model.eval()

    @torch.no_grad()
    def predict_class(self, input_ids) -> int:
        ids = torch.as_tensor(input_ids, dtype=torch.long, device=next(self.model.parameters()).device)
        if ids.dim() == 1:
            ids = ids[None]
        return int(self.model(ids)[0].argmax())

    @torch.no_grad()
    def predict_proba(self, input_ids) -> torch.Tensor:
        ids = torch.as_tensor(input_ids, dtype=torch.long, device=next(self.model.parameters()).device)
        return torch.softmax(self.model(ids if ids.dim() == 2 else ids[None]).float(), -1)


class TextGenerationPipeline:
    """GptLite text generation from a prompt of token ids with the sampling settings of
    ``GenerationConfig`` (repetition penalty, temperature, top-k / top-p / min-p)."""

    def __init__(self, config: GptLiteConfig, seed: int = 0, device=None, model=None):
        from .families import GptLite
        self.model = model or GptLite(config, device=device, seed=seed)
        self.model.eval()

    @torch.no_grad()
    def generate(self, prompt_ids, config: GenerationConfig | None = None) -> list[int]:
        ids = torch.as_tensor(prompt_ids, dtype=torch.long, device=next(self.model.parameters()).device)
        out = self.model.generate(ids if ids.dim() == 2 else ids[None], config)
        return out[0].tolist()
