"""Plain-PyTorch baseline of the headline training benchmark: the Llama-3-8B-shaped model written with
eager torch modules and nothing from this framework.

- GEMMs through ``nn.Linear`` (cuBLAS), attention through ``F.scaled_dot_product_attention``
  (causal, grouped-query; PyTorch picks its fastest fused backend), RMSNorm as ``nn.RMSNorm``,
  RoPE (NeoX half rotation) and SwiGLU as torch elementwise ops, the LM head and mean
  cross-entropy with ``F.cross_entropy``;
- bf16 parameters and gradients, ``torch.optim.AdamW(fused=True)`` (its moments follow the
  parameter dtype, so this baseline moves fewer optimizer bytes than the framework's f32 master
  weights and moments);
- ``torch.nn.parallel.DistributedDataParallel`` over NCCL when there is more than one rank.

``bench.py --impl torch`` times it with the same rules as the framework's arm (warm-up, CUDA events,
max over ranks, clocks, an end-to-end loop with host-to-device input copies and the loss read back).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class _Block(nn.Module):
    def __init__(self, d, hq, hkv, hd, ffn, eps):
        super().__init__()
        self.hq, self.hkv, self.hd = hq, hkv, hd
        self.attn_norm = nn.RMSNorm(d, eps=eps)
        self.wqkv = nn.Linear(d, (hq + 2 * hkv) * hd, bias=False)
        self.wo = nn.Linear(hq * hd, d, bias=False)
        self.ffn_norm = nn.RMSNorm(d, eps=eps)
        self.w_gate_up = nn.Linear(d, 2 * ffn, bias=False)
        self.w_down = nn.Linear(ffn, d, bias=False)

    @staticmethod
    def _rope(x, cos, sin):
        half = x.shape[-1] // 2
        rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
        return x * cos + rot * sin

    def forward(self, x, cos, sin):
        B, S, _ = x.shape
        qkv = self.wqkv(self.attn_norm(x)).view(B, S, self.hq + 2 * self.hkv, self.hd)
        q, k, v = qkv.split([self.hq, self.hkv, self.hkv], dim=2)
        q = self._rope(q.transpose(1, 2), cos, sin)
        k = self._rope(k.transpose(1, 2), cos, sin)
        o = F.scaled_dot_product_attention(q, k, v.transpose(1, 2), is_causal=True, enable_gqa=True)
        x = x + self.wo(o.transpose(1, 2).reshape(B, S, -1))
        g, u = self.w_gate_up(self.ffn_norm(x)).chunk(2, dim=-1)
        return x + self.w_down(F.silu(g) * u)


class TorchLlama(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        d, hd = cfg.hidden_dim, cfg.head_dim
        self.embed = nn.Embedding(cfg.vocab_size, d)
        self.blocks = nn.ModuleList(_Block(d, cfg.num_heads, cfg.num_kv_heads, hd, cfg.intermediate_dim, cfg.norm_eps)
                                    for _ in range(cfg.num_layers))
        self.norm = nn.RMSNorm(d, eps=cfg.norm_eps)
        self.head = nn.Linear(d, cfg.vocab_size, bias=False)

    def rope_tables(self, S, device):
        hd = self.cfg.head_dim
        inv = 1.0 / (self.cfg.rope_theta ** (torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd))
        ang = torch.outer(torch.arange(S, device=device, dtype=torch.float32), inv)
        ang = torch.cat([ang, ang], dim=-1)
        return ang.cos().bfloat16(), ang.sin().bfloat16()

    def forward(self, tokens, targets, cos, sin):
        x = self.embed(tokens)
        for blk in self.blocks:
            x = blk(x, cos, sin)
        logits = self.head(self.norm(x))
        return F.cross_entropy(logits.view(-1, logits.shape[-1]).float(), targets.reshape(-1))


def build(cfg, device, seed=0):
    """The model in bf16 on `device`, every weight N(0, 0.02) (norm gains 1), seeded."""
    torch.manual_seed(seed)
    with torch.device(device):
        model = TorchLlama(cfg).to(torch.bfloat16)
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.fill_(1.0)
            else:
                p.normal_(0.0, 0.02, generator=g)
    return model
