"""Model configurations with the reference's field names, plus the benchmark presets.

``LlamaLiteConfig`` mirrors crates/brain-transformer/src/models/llama_lite.rs:24-60 (vocab_size,
hidden_dim, num_layers, num_heads, num_kv_heads, head_dim, intermediate_dim, max_seq_len,
rope_theta, norm_eps); ``GptLiteConfig`` mirrors gpt_lite.rs:24-60; ``BertLiteConfig`` and
``T5LiteConfig`` mirror bert_lite.rs / t5_lite.rs; ``ViTConfig`` mirrors brain-vit's ViT-B defaults
(crates/brain-vit/src/vit/mod.rs:132). ``TransformerConfig`` presets follow
crates/brain-transformer/src/config/mod.rs (bert_base, gpt2_small, llama_7b).
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass


@dataclass
class LlamaLiteConfig:
    vocab_size: int = 32000
    hidden_dim: int = 512
    num_layers: int = 4
    num_heads: int = 8
    num_kv_heads: int = 8
    head_dim: int = 64
    intermediate_dim: int = 1376
    max_seq_len: int = 2048
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    tie_embeddings: bool = False
    init_std: float = 0.02

    @staticmethod
    def llama3_8b(max_seq_len: int = 8192) -> "LlamaLiteConfig":
        return LlamaLiteConfig(vocab_size=128256, hidden_dim=4096, num_layers=32, num_heads=32, num_kv_heads=8,
                               head_dim=128, intermediate_dim=14336, max_seq_len=max_seq_len, rope_theta=500000.0,
                               norm_eps=1e-5)

    @staticmethod
    def llama3_70b(max_seq_len: int = 8192) -> "LlamaLiteConfig":
        return LlamaLiteConfig(vocab_size=128256, hidden_dim=8192, num_layers=80, num_heads=64, num_kv_heads=8,
                               head_dim=128, intermediate_dim=28672, max_seq_len=max_seq_len, rope_theta=500000.0,
                               norm_eps=1e-5)

    @staticmethod
    def tiny(vocab_size=256, layers=2) -> "LlamaLiteConfig":
        return LlamaLiteConfig(vocab_size=vocab_size, hidden_dim=128, num_layers=layers, num_heads=4, num_kv_heads=2,
                               head_dim=32, intermediate_dim=256, max_seq_len=256)

    def replace(self, **kw):
        return dataclasses.replace(self, **kw)

    def num_params(self) -> int:
        d, f, v = self.hidden_dim, self.intermediate_dim, self.vocab_size
        qkv = d * (self.num_heads + 2 * self.num_kv_heads) * self.head_dim
        o = self.num_heads * self.head_dim * d
        per_layer = qkv + o + 3 * d * f + 2 * d
        head = 0 if self.tie_embeddings else v * d
        return v * d + self.num_layers * per_layer + d + head


@dataclass
class GptLiteConfig:
    vocab_size: int = 1024
    hidden_dim: int = 128
    num_layers: int = 2
    num_heads: int = 4
    intermediate_dim: int = 512
    max_seq_len: int = 64
    norm_eps: float = 1e-5
    bias: bool = True
    tie_embeddings: bool = False
    init_std: float = 0.02

    @staticmethod
    def lite_2x128() -> "GptLiteConfig":
        """2 layers, d 128, 4 heads, FFN 512 GELU, LN, learned positions, vocab 1024, seq 64."""
        return GptLiteConfig()

    @staticmethod
    def gpt2_small() -> "GptLiteConfig":
        return GptLiteConfig(vocab_size=50257, hidden_dim=768, num_layers=12, num_heads=12, intermediate_dim=3072,
                             max_seq_len=1024, tie_embeddings=True)


@dataclass
class BertLiteConfig:
    vocab_size: int = 30522
    hidden_dim: int = 256
    num_layers: int = 4
    num_heads: int = 4
    intermediate_dim: int = 1024
    max_seq_len: int = 512
    type_vocab_size: int = 2
    norm_eps: float = 1e-12
    num_labels: int = 2

    @staticmethod
    def bert_base() -> "BertLiteConfig":
        return BertLiteConfig(hidden_dim=768, num_layers=12, num_heads=12, intermediate_dim=3072)


@dataclass
class T5LiteConfig:
    vocab_size: int = 32128
    hidden_dim: int = 256
    num_layers: int = 4
    num_decoder_layers: int = 4
    num_heads: int = 4
    intermediate_dim: int = 1024
    max_seq_len: int = 512
    relative_buckets: int = 32
    max_distance: int = 128
    norm_eps: float = 1e-6


@dataclass
class ViTConfig:
    image_size: int = 224
    patch_size: int = 16
    in_channels: int = 3
    hidden_dim: int = 768
    num_layers: int = 12
    num_heads: int = 12
    mlp_dim: int = 3072
    num_classes: int = 1000
    norm_eps: float = 1e-6

    @staticmethod
    def vit_b16() -> "ViTConfig":
        return ViTConfig()

    @property
    def num_patches(self) -> int:
        return (self.image_size // self.patch_size) ** 2


@dataclass
class TransformerConfig:
    """Generic encoder/decoder description used by the builder (config/mod.rs presets)."""
    vocab_size: int = 32000
    hidden_dim: int = 512
    num_layers: int = 6
    num_heads: int = 8
    num_kv_heads: int = 8
    intermediate_dim: int = 2048
    max_seq_len: int = 512
    norm: str = "rms"          # "rms" | "layer"
    activation: str = "swiglu"  # "swiglu" | "gelu"
    pre_norm: bool = True
    causal: bool = True
    rope: bool = True
    learned_positions: bool = False
    bias: bool = False
    norm_eps: float = 1e-5
    rope_theta: float = 10000.0

    @staticmethod
    def bert_base():
        return TransformerConfig(30522, 768, 12, 12, 12, 3072, 512, "layer", "gelu", False, False, False, True, True,
                                 1e-12)

    @staticmethod
    def gpt2_small():
        return TransformerConfig(50257, 768, 12, 12, 12, 3072, 1024, "layer", "gelu", True, True, False, True, True)

    @staticmethod
    def llama_7b():
        return TransformerConfig(32000, 4096, 32, 32, 32, 11008, 4096, "rms", "swiglu", True, True, True, False,
                                 False, 1e-5)
