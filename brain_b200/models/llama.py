"""LlamaLite: pre-norm decoder with RMSNorm, GQA, RoPE and SwiGLU, on the sm_100a kernels.

API parity with crates/brain-transformer/src/models/llama_lite.rs:24-187 (``LlamaLite::new(config)``,
``forward``, ``generate``), with the reference's gaps closed on purpose: the decoder really uses
``num_kv_heads`` (grouped-query attention) and really applies RoPE (theta from the config), and
``generate`` decodes incrementally from a KV cache instead of re-running the whole prefix.

Each block is four fused ops:
    qkv = norm_linear(h, attn_norm, Wqkv, rope)           RMSNorm recomputed in backward, RoPE in the GEMM epilogue
    h   = linear(qkv_attention(qkv), Wo, +h)              flash attention, residual epilogue
    gu  = norm_linear(h, ffn_norm, Wgate_up)
    h   = swiglu_linear(gu, Wdown, +h)                    SwiGLU recomputed in backward
and the LM head is a fused linear + cross-entropy.
"""
from __future__ import annotations

import torch

from .. import ops
from ..nn import init as _init
from ..nn.module import Module, ModuleList
from .config import LlamaLiteConfig
from .generate import GenerationConfig, sample_next_token
from .kv_cache import KvCache, KvCacheConfig


class LlamaBlock(Module):
    def __init__(self, cfg: LlamaLiteConfig, device=None, dtype=None):
        super().__init__()
        d, hd = cfg.hidden_dim, cfg.head_dim
        self.cfg = cfg
        self.attn_norm = torch.nn.Parameter(torch.ones(d, device=device, dtype=dtype))
        self.wqkv = torch.nn.Parameter(torch.empty((cfg.num_heads + 2 * cfg.num_kv_heads) * hd, d, device=device,
                                                   dtype=dtype))
        self.wo = torch.nn.Parameter(torch.empty(d, cfg.num_heads * hd, device=device, dtype=dtype))
        self.ffn_norm = torch.nn.Parameter(torch.ones(d, device=device, dtype=dtype))
        self.w_gate_up = torch.nn.Parameter(torch.empty(2 * cfg.intermediate_dim, d, device=device, dtype=dtype))
        self.w_down = torch.nn.Parameter(torch.empty(d, cfg.intermediate_dim, device=device, dtype=dtype))

    def forward(self, h, rope, cache: KvCache | None = None, layer: int = 0, pos: int = 0):
        c = self.cfg
        if cache is None:
            # RoPE on the q and k heads in the QKV GEMM's epilogue; attention gets them rotated
            qkv = ops.norm_linear(h, self.attn_norm, self.wqkv, c.norm_eps,
                                  rope=(rope, c.num_heads + c.num_kv_heads, c.head_dim, h.shape[-2], 0))
            o = ops.qkv_attention(qkv, c.num_heads, c.num_kv_heads, None)
        else:
            qkv = ops.norm_linear(h, self.attn_norm, self.wqkv, c.norm_eps)
            o = self._cached_attention(qkv, rope, cache, layer, pos)
        h = ops.linear(o, self.wo, residual=h)
        gu = ops.norm_linear(h, self.ffn_norm, self.w_gate_up, c.norm_eps)
        return ops.swiglu_linear(gu, self.w_down, residual=h)

    def _cached_attention(self, qkv, rope, cache, layer, pos):
        c = self.cfg
        q, k, v = ops.attention.split_qkv(qkv, c.num_heads, c.num_kv_heads)
        if q.is_cuda:
            ops.apply_rope_(q, rope, offset=pos)
            ops.apply_rope_(k, rope, offset=pos)
        else:
            q = ops.rope.rope_ref(q, rope, None, pos)
            k = ops.rope.rope_ref(k, rope, None, pos)
        kf, vf = cache.update(layer, k, v)
        if q.is_cuda:
            o, _ = ops.flash_attention_fwd(q, kf, vf, causal=True)
        else:
            o = ops.sdpa_ref(q, kf, vf, causal=True)
        return o.reshape(qkv.shape[0], qkv.shape[1], -1)


class LlamaLite(Module):
    def __init__(self, config: LlamaLiteConfig, device=None, dtype=torch.bfloat16, seed: int = 0, init: bool = True):
        super().__init__()
        self.config = config
        c = config
        self.embed = torch.nn.Parameter(torch.empty(c.vocab_size, c.hidden_dim, device=device, dtype=dtype))
        self.layers = ModuleList([LlamaBlock(c, device, dtype) for _ in range(c.num_layers)])
        self.final_norm = torch.nn.Parameter(torch.ones(c.hidden_dim, device=device, dtype=dtype))
        self.lm_head = None if c.tie_embeddings else torch.nn.Parameter(
            torch.empty(c.vocab_size, c.hidden_dim, device=device, dtype=dtype))
        self.activation_checkpointing = False
        if init:
            _init.init_normal_(self, c.init_std, seed)

    # ------------------------------------------------------------------ helpers
    def head_weight(self):
        return self.embed if self.lm_head is None else self.lm_head

    def rope(self, device, length=None):
        c = self.config
        return ops.rope_table(c.head_dim, length or c.max_seq_len, c.rope_theta, device=device)

    def hidden(self, tokens: torch.Tensor, cache: KvCache | None = None, pos: int = 0) -> torch.Tensor:
        c = self.config
        rope = self.rope(tokens.device, max(c.max_seq_len, pos + tokens.shape[1]))
        h = ops.embedding(tokens, self.embed)
        for i, blk in enumerate(self.layers):
            if self.activation_checkpointing and self.training and cache is None:
                h = torch.utils.checkpoint.checkpoint(blk, h, rope, use_reentrant=False)
            else:
                h = blk(h, rope, cache, i, pos)
        return h

    # ------------------------------------------------------------------ public API
    def forward(self, tokens: torch.Tensor, cache: KvCache | None = None, pos: int = 0) -> torch.Tensor:
        """tokens [B, S] -> logits [B, S, V]."""
        h = self.hidden(tokens, cache, pos)
        h = ops.rms_norm(h, self.final_norm, self.config.norm_eps)
        return ops.linear(h, self.head_weight())

    def loss(self, tokens: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
        """Mean next-token cross-entropy; the LM head and the loss run fused."""
        h = self.hidden(tokens)
        h = ops.rms_norm(h, self.final_norm, self.config.norm_eps)
        return ops.linear_cross_entropy(h, self.head_weight(), labels, ignore_index)

    def make_cache(self, batch_size: int, max_len: int | None = None) -> KvCache:
        c = self.config
        dev = self.embed.device
        return KvCache(KvCacheConfig(c.num_layers, batch_size, c.num_kv_heads, c.head_dim,
                                     max_len or c.max_seq_len, self.embed.dtype, dev))

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, cfg: GenerationConfig | None = None) -> torch.Tensor:
        """prompt [B, S] -> [B, S + new] (prefill once, then one token per step from the KV cache)."""
        cfg = cfg or GenerationConfig()
        B, S = prompt.shape
        cache = self.make_cache(B, S + cfg.max_new_tokens)
        gen = torch.Generator(device=prompt.device).manual_seed(cfg.seed)
        logits = self.forward(prompt, cache, 0)[:, -1]
        out = [prompt]
        history = prompt
        done = torch.zeros(B, dtype=torch.bool, device=prompt.device)
        for t in range(cfg.max_new_tokens):
            nxt = sample_next_token(logits, cfg, history, gen)
            if cfg.eos_token_id is not None:
                nxt = torch.where(done, torch.full_like(nxt, cfg.eos_token_id), nxt)
                done |= nxt == cfg.eos_token_id
            out.append(nxt[:, None])
            history = torch.cat([history, nxt[:, None]], 1)
            if t + 1 == cfg.max_new_tokens or (cfg.eos_token_id is not None and bool(done.all())):
                break
            logits = self.forward(nxt[:, None], cache, S + t)[:, -1]
        return torch.cat(out, 1)
