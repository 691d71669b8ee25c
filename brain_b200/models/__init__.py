"""Model families: LlamaLite (GQA + RoPE + SwiGLU), GptLite, BertLite, T5Lite, ViT."""
from .config import LlamaLiteConfig, GptLiteConfig, BertLiteConfig, T5LiteConfig, ViTConfig, TransformerConfig  # noqa: F401
from .llama import LlamaLite, LlamaBlock  # noqa: F401
from .kv_cache import KvCache, KvCacheConfig, PagedKvCache  # noqa: F401
from .generate import GenerationConfig, sample_next_token  # noqa: F401
from .families import GptLite, BertLite, T5Lite, ViT  # noqa: F401
VitModel = ViT  # the reference's name (crates/brain-vit/src/impl.rs)
from .blocks import TransformerBlock, TransformerStack  # noqa: F401
from .transformer_api import (FlashAttentionLite, FlashLiteConfig, XformersAttentionLite, XformersConfig,  # noqa: F401
                              RelativeAttention, AlibiPositionalBias, LayerKvCache, TransformerDecoderLayer,
                              TransformerDecoder, repeat_kv, quick_gelu, all_close,
                              TransformerEncoder, TransformerEncoderLayer, EncoderLayer, TransformerEncoderBlock,
                              build_encoder, build_decoder, RopeConfig, RotaryEmbedding, PositionalEncoding,
                              RelativePositionBias, split_heads, merge_heads)
