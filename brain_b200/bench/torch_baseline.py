"""Plain-PyTorch baseline of the headline training benchmark: the Llama-3-8B-shaped model written with
eager torch modules and nothing from this framework.

- GEMMs through ``nn.Linear`` (cuBLAS), attention through ``F.scaled_dot_product_attention``
  (causal, grouped-query; PyTorch picks its fastest fused backend), RMSNorm as ``nn.RMSNorm``,
  RoPE (NeoX half rotation) and SwiGLU as torch elementwise ops, the LM head and mean
  cross-entropy with ``F.cross_entropy``;
- bf16 parameters and gradients; the optimizer is either ``torch.optim.AdamW(fused=True)`` on the bf16
  parameters (its moments follow the parameter dtype: fewer optimizer bytes than the framework's) or,
  with ``--torch-master fp32``, :class:`MasterAdamW`: float32 master weights and moments, ZeRO-1
  sharded over the ranks, the same precision as the framework's sharded AdamW;
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
    """The model in bf16 on `device`, seeded exactly like the framework's ``LlamaLite(cfg, seed=seed)``:
    one generator on the device walks the weight matrices in LlamaLite's parameter order (embedding, LM
    head, then per block wqkv, wo, w_gate_up, w_down; the same shapes) and draws float32 N(0, 0.02)
    samples rounded to bf16; norm gains are 1. Both arms therefore start
    from identical weights, and their loss trajectories on identical data can be compared directly."""
    torch.manual_seed(seed)
    with torch.device(device):
        model = TorchLlama(cfg).to(torch.bfloat16)
    g = torch.Generator(device=device).manual_seed(seed)
    # LlamaLite's parameter order: its own tensors (embedding, final norm, LM head) before the blocks'
    order = [model.embed.weight, model.head.weight]
    for blk in model.blocks:
        order += [blk.wqkv.weight, blk.wo.weight, blk.w_gate_up.weight, blk.w_down.weight]
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() < 2:
                p.fill_(1.0)
        for p in order:
            p.copy_((torch.randn(p.shape, generator=g, device=p.device, dtype=torch.float32) * cfg.init_std)
                    .to(p.dtype))
    return model


class MasterAdamW:
    """AdamW on float32 master weights and float32 moments for a bf16 model, in plain PyTorch.

    Gradients arrive in bf16 on the model's parameters (DDP reduces them there). Each step casts them to
    float32 in chunks of parameters (so at most one chunk of float32 gradients exists at a time), runs
    ``torch.optim.AdamW(fused=True)`` on the chunk's master weights and copies the result back to the
    bf16 parameters. With ``world > 1`` the optimizer state is sharded ZeRO-1 style: parameters are dealt
    round-robin by size to ranks, each rank steps only its own, and the updated bf16 weights are
    broadcast from their owners (one NCCL broadcast per parameter, coalesced by torch)."""

    def __init__(self, params, lr, betas, eps, weight_decay, world=1, rank=0, chunk_bytes=2 << 30):
        import torch.distributed as dist
        self.params = [p for p in params if p.requires_grad]
        self.world, self.rank = world, rank
        owners, load = [], [0] * world
        for p in sorted(self.params, key=lambda t: -t.numel()):
            r = min(range(world), key=lambda i: load[i])
            owners.append((p, r))
            load[r] += p.numel()
        self.owner = {id(p): r for p, r in owners}
        mine = [p for p in self.params if self.owner[id(p)] == rank]
        self.master = {id(p): torch.nn.Parameter(p.detach().float().clone()) for p in mine}
        self.chunks, cur, size = [], [], 0
        for p in mine:
            cur.append(p)
            size += p.numel() * 4
            if size >= chunk_bytes:
                self.chunks.append(cur)
                cur, size = [], 0
        if cur:
            self.chunks.append(cur)
        self.opts = [torch.optim.AdamW([self.master[id(p)] for p in c], lr=lr, betas=betas, eps=eps,
                                       weight_decay=weight_decay, fused=True) for c in self.chunks]
        self._dist = dist

    @torch.no_grad()
    def step(self):
        for chunk, opt in zip(self.chunks, self.opts):
            for p in chunk:
                self.master[id(p)].grad = p.grad.float()
            opt.step()
            for p in chunk:
                m = self.master[id(p)]
                m.grad = None
                p.copy_(m)
        if self.world > 1:
            for p in self.params:
                self._dist.broadcast(p.data, self.owner[id(p)])

    def zero_grad(self, set_to_none=False):
        for p in self.params:
            if p.grad is not None:
                if set_to_none:
                    p.grad = None
                else:
                    p.grad.zero_()


class _VitBlock(nn.Module):
    """Pre-norm encoder block: LayerNorm, fused-QKV attention through F.scaled_dot_product_attention, tanh
    GELU MLP; every Linear with a bias (cuBLAS)."""

    def __init__(self, d, heads, mlp, eps, device, dtype):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.heads = heads
        self.n1 = nn.LayerNorm(d, eps=eps, **kw)
        self.qkv = nn.Linear(d, 3 * d, **kw)
        self.proj = nn.Linear(d, d, **kw)
        self.n2 = nn.LayerNorm(d, eps=eps, **kw)
        self.fc1 = nn.Linear(d, mlp, **kw)
        self.fc2 = nn.Linear(mlp, d, **kw)

    def forward(self, x):
        B, S, D = x.shape
        q, k, v = self.qkv(self.n1(x)).view(B, S, 3, self.heads, D // self.heads).permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(q, k, v)
        x = x + self.proj(o.transpose(1, 2).reshape(B, S, D))
        return x + self.fc2(F.gelu(self.fc1(self.n2(x)), approximate="tanh"))


class TorchViT(nn.Module):
    """ViT-B/16 in plain PyTorch for the comparison arm: patch embedding as one Linear over the 16x16
    patches (a stride-16 convolution), class token, learned positions, 12 pre-norm blocks, final
    LayerNorm, linear head on the class token; the same architecture as ``models.families.ViT``."""

    def __init__(self, cfg, device, dtype=torch.bfloat16):
        super().__init__()
        self.cfg = cfg
        P, d = cfg.patch_size, cfg.hidden_dim
        kw = dict(device=device, dtype=dtype)
        self.patch = nn.Linear(cfg.in_channels * P * P, d, **kw)
        self.cls_token = nn.Parameter(torch.zeros(1, 1, d, **kw))
        self.pos = nn.Parameter(torch.zeros(1, cfg.num_patches + 1, d, **kw))
        self.blocks = nn.ModuleList([_VitBlock(d, cfg.num_heads, cfg.mlp_dim, cfg.norm_eps, device, dtype)
                                     for _ in range(cfg.num_layers)])
        self.norm = nn.LayerNorm(d, eps=cfg.norm_eps, **kw)
        self.head = nn.Linear(d, cfg.num_classes, **kw)
        g = torch.Generator(device="cpu").manual_seed(0)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if p.dim() >= 2 or name in ("cls_token", "pos"):
                    p.copy_((torch.randn(p.shape, generator=g) * 0.02).to(dtype))

    def forward(self, images, labels):
        B, C, H, W = images.shape
        P = self.cfg.patch_size
        x = images.reshape(B, C, H // P, P, W // P, P).permute(0, 2, 4, 1, 3, 5).reshape(B, -1, C * P * P)
        x = self.patch(x)
        x = torch.cat([self.cls_token.expand(B, -1, -1), x], 1) + self.pos
        for blk in self.blocks:
            x = blk(x)
        logits = self.head(self.norm(x)[:, 0])
        return F.cross_entropy(logits.float(), labels)
