"""GPT-lite, BERT-lite, T5-lite and ViT on the shared blocks.

* ``GptLite`` (crates/brain-transformer/src/models/gpt_lite.rs:24-171): token + learned position
  embedding followed by an embedding LayerNorm, pre-LN causal decoder with tanh-GELU FFN, final
  norm, bias-free LM head. The 2-layer, d 128 data-parallel training workload uses ``GptLiteConfig.lite_2x128()``.
* ``BertLite`` (bert_lite.rs:23-200): token + position + token-type embeddings with LayerNorm,
  post-LN bidirectional encoder, tanh pooler over [CLS], classification head, optional MLM head.
* ``T5Lite`` (t5_lite.rs:25-200): RMSNorm pre-norm encoder/decoder with bucketed relative position
  bias (attention/relative.rs), cross-attention, ReLU FFN, tied embedding scaling.
* ``ViT`` (brain-vit ViT-B/16 defaults, crates/brain-vit/src/vit/mod.rs:132): patch embedding as a
  reshape + GEMM (patch 16, stride 16 is a pure reshape), [CLS] token, learned positions,
  pre-LN encoder with GELU MLP, classification head on [CLS].
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..nn import init as _init
from ..nn.layers import Embedding, LayerNorm, Linear
from ..nn.module import Module
from .blocks import TransformerStack, make_norm
from .config import BertLiteConfig, GptLiteConfig, T5LiteConfig, ViTConfig
from .generate import GenerationConfig, sample_next_token


class GptLite(Module):
    def __init__(self, config: GptLiteConfig, device=None, dtype=torch.float32, seed: int = 0, init: bool = True):
        super().__init__()
        c = self.config = config
        self.tok = torch.nn.Parameter(torch.empty(c.vocab_size, c.hidden_dim, device=device, dtype=dtype))
        self.pos = torch.nn.Parameter(torch.empty(c.max_seq_len, c.hidden_dim, device=device, dtype=dtype))
        self.emb_norm = LayerNorm(c.hidden_dim, c.norm_eps, True, device, dtype)
        self.decoder = TransformerStack(c.num_layers, c.hidden_dim, c.num_heads, c.intermediate_dim, norm="layer",
                                        act="gelu", pre_norm=True, causal=True, bias=c.bias, eps=c.norm_eps,
                                        device=device, dtype=dtype)
        self.lm_head = None if c.tie_embeddings else torch.nn.Parameter(
            torch.empty(c.vocab_size, c.hidden_dim, device=device, dtype=dtype))
        if init:
            _init.init_normal_(self, c.init_std, seed)

    def head_weight(self):
        return self.tok if self.lm_head is None else self.lm_head

    def hidden(self, ids):
        S = ids.shape[-1]
        if S > self.config.max_seq_len:
            raise ValueError("sequence longer than max_seq_len")
        h = ops.embedding(ids, self.tok, self.pos[:S].contiguous() if ids.is_cuda else self.pos[:S])
        return self.decoder(self.emb_norm(h))

    def forward(self, ids):
        return ops.linear(self.hidden(ids), self.head_weight())

    def loss(self, ids, labels, ignore_index=-100):
        return ops.linear_cross_entropy(self.hidden(ids), self.head_weight(), labels, ignore_index)

    @torch.no_grad()
    def generate(self, prompt, cfg: GenerationConfig | None = None):
        cfg = cfg or GenerationConfig()
        out = prompt
        g = torch.Generator(device=prompt.device).manual_seed(cfg.seed)
        for _ in range(cfg.max_new_tokens):
            if out.shape[1] >= self.config.max_seq_len:
                break
            nxt = sample_next_token(self.forward(out)[:, -1], cfg, out, g)
            out = torch.cat([out, nxt[:, None]], 1)
        return out


class BertLite(Module):
    def __init__(self, config: BertLiteConfig, device=None, dtype=torch.float32, seed: int = 0):
        super().__init__()
        c = self.config = config
        self.tok = Embedding(c.vocab_size, c.hidden_dim, device, dtype)
        self.pos = Embedding(c.max_seq_len, c.hidden_dim, device, dtype)
        self.typ = Embedding(c.type_vocab_size, c.hidden_dim, device, dtype)
        self.emb_norm = LayerNorm(c.hidden_dim, c.norm_eps, True, device, dtype)
        self.encoder = TransformerStack(c.num_layers, c.hidden_dim, c.num_heads, c.intermediate_dim, final_norm=False,
                                        norm="layer", act="gelu", pre_norm=False, causal=False, bias=True,
                                        eps=c.norm_eps, device=device, dtype=dtype)
        self.pooler = Linear(c.hidden_dim, c.hidden_dim, True, device, dtype)
        self.cls = Linear(c.hidden_dim, c.num_labels, True, device, dtype)
        self.mlm = Linear(c.hidden_dim, c.vocab_size, True, device, dtype)
        _init.init_normal_(self, 0.02, seed)

    def encode(self, ids, token_type=None, attention_mask=None):
        B, S = ids.shape
        pos = torch.arange(S, device=ids.device)[None].expand(B, S)
        tt = token_type if token_type is not None else torch.zeros_like(ids)
        h = self.tok(ids) + self.pos(pos) + self.typ(tt)
        return self.encoder(self.emb_norm(h), mask=attention_mask)

    def forward(self, ids, token_type=None, attention_mask=None):
        h = self.encode(ids, token_type, attention_mask)
        pooled = torch.tanh(self.pooler(h[:, 0]))
        return self.cls(pooled)

    def mlm_logits(self, ids, token_type=None, attention_mask=None):
        return self.mlm(self.encode(ids, token_type, attention_mask))


def relative_position_bucket(rel: torch.Tensor, bidirectional: bool, num_buckets: int, max_distance: int):
    """T5 bucketing: exact buckets for small distances, logarithmic ones up to max_distance."""
    ret = torch.zeros_like(rel)
    n = -rel
    if bidirectional:
        num_buckets //= 2
        ret = ret + (n < 0).long() * num_buckets
        n = n.abs()
    else:
        n = n.clamp_min(0)
    max_exact = num_buckets // 2
    is_small = n < max_exact
    large = max_exact + (torch.log(n.float().clamp_min(1) / max_exact) / math.log(max_distance / max_exact)
                         * (num_buckets - max_exact)).long()
    large = large.clamp_max(num_buckets - 1)
    return ret + torch.where(is_small, n, large)


class T5Lite(Module):
    def __init__(self, config: T5LiteConfig, device=None, dtype=torch.float32, seed: int = 0):
        super().__init__()
        c = self.config = config
        self.shared = Embedding(c.vocab_size, c.hidden_dim, device, dtype)
        kw = dict(norm="rms", act="relu", pre_norm=True, bias=False, eps=c.norm_eps, device=device, dtype=dtype)
        self.encoder = TransformerStack(c.num_layers, c.hidden_dim, c.num_heads, c.intermediate_dim, causal=False, **kw)
        self.decoder = TransformerStack(c.num_decoder_layers, c.hidden_dim, c.num_heads, c.intermediate_dim,
                                        causal=True, cross=True, **kw)
        self.enc_bias = torch.nn.Parameter(torch.zeros(c.relative_buckets, c.num_heads, device=device, dtype=dtype))
        self.dec_bias = torch.nn.Parameter(torch.zeros(c.relative_buckets, c.num_heads, device=device, dtype=dtype))
        _init.init_normal_(self, 0.02, seed)

    def _bias(self, table, Sq, Sk, bidirectional, device):
        """The bucketed bias as a function of the key-query offset k - q (``RelativeBias``, [H, Sq + Sk - 1]):
        the masked flash kernels read it directly when it needs no gradient."""
        from ..ops.attention import RelativeBias
        c = self.config
        rel = torch.arange(-(Sq - 1), Sk, device=device)
        b = relative_position_bucket(rel, bidirectional, c.relative_buckets, c.max_distance)
        return RelativeBias(table[b].t().float(), Sq, Sk)  # [H, Sq + Sk - 1]

    def forward(self, src_ids, tgt_ids):
        Ss, St = src_ids.shape[1], tgt_ids.shape[1]
        mem = self.encoder(self.shared(src_ids), attn_bias=self._bias(self.enc_bias, Ss, Ss, True, src_ids.device))
        h = self.decoder(self.shared(tgt_ids), attn_bias=self._bias(self.dec_bias, St, St, False, tgt_ids.device),
                         mem=mem)
        return ops.linear(h * (self.config.hidden_dim ** -0.5), self.shared.weight)


class ViT(Module):
    def __init__(self, config: ViTConfig, device=None, dtype=torch.float32, seed: int = 0):
        super().__init__()
        c = self.config = config
        P = c.patch_size
        self.patch = Linear(c.in_channels * P * P, c.hidden_dim, True, device, dtype)
        self.cls_token = torch.nn.Parameter(torch.zeros(1, 1, c.hidden_dim, device=device, dtype=dtype))
        self.pos = torch.nn.Parameter(torch.zeros(1, c.num_patches + 1, c.hidden_dim, device=device, dtype=dtype))
        self.encoder = TransformerStack(c.num_layers, c.hidden_dim, c.num_heads, c.mlp_dim, norm="layer", act="gelu",
                                        pre_norm=True, causal=False, bias=True, eps=c.norm_eps, device=device,
                                        dtype=dtype)
        self.head = Linear(c.hidden_dim, c.num_classes, True, device, dtype)
        _init.init_normal_(self, 0.02, seed)

    def patchify(self, images):
        """[B, C, H, W] -> [B, N, C*P*P] (stride == patch, so a pure reshape)."""
        B, C, H, W = images.shape
        P = self.config.patch_size
        x = images.reshape(B, C, H // P, P, W // P, P).permute(0, 2, 4, 1, 3, 5)
        return x.reshape(B, (H // P) * (W // P), C * P * P)

    def embed_patches(self, images):
        """[B, C, H, W] -> [B, 1 + N, D]: patch projection (one GEMM), class token, position embedding."""
        x = self.patch(self.patchify(images).to(self.patch.weight.dtype))
        cls = self.cls_token.expand(x.shape[0], -1, -1)
        return torch.cat([cls, x], 1) + self.pos

    def forward_features(self, images):
        """Encoder output for every token [B, 1 + N, D] (class token first)."""
        return self.encoder(self.embed_patches(images))

    def forward(self, images):
        return self.head(self.forward_features(images)[:, 0])

    def loss(self, images, labels):
        return ops.cross_entropy(self.forward(images), labels)
