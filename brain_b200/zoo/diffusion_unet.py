"""Diffusion U-Net, pseudo-linear-multistep sampling, conditioning and a training loop.

Reference: crates/brain-diffusion/src/unet/ (UnetConfig, Unet2d, ResBlock, SpatialTransformer,
Downsample2d, Upsample2d, sinusoidal embeddings), samplers/plms.rs (PlmsSampler), guidance.rs
(apply_cfg), conditioning.rs (ConditioningContext), diffusion/train.rs (DiffusionTrainer),
latent.rs (IdentityLatentCodec). The reference's ``Unet2d::forward`` returns zeros and its PLMS
step returns x unchanged; here the U-Net is the usual time-conditioned encoder-decoder (residual
blocks with GroupNorm/SiLU and a timestep projection, self- and cross-attention transformers at
the lower resolutions, stride-2 downsampling, nearest upsampling, skip concatenation) and PLMS is
the 4th-order Adams-Bashforth update on epsilon of Liu et al. 2022 (lower orders for the first
steps). Attention runs through ``F.scaled_dot_product_attention`` so fused kernels apply on a GPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .diffusion import NoiseSchedule, diffusion_loss, guided_eps, timestep_embedding


@dataclass
class UnetConfig:
    in_channels: int = 4
    out_channels: int = 4
    model_channels: int = 64
    num_res_blocks: int = 2
    channel_mult: tuple = (1, 2, 4)
    attention_levels: tuple = (1, 2)  # resolution levels with a SpatialTransformer
    num_heads: int = 4
    context_dim: int | None = None  # cross-attention width (None: self-attention only)
    groups: int = 32


def _gn(c: int, groups: int) -> nn.GroupNorm:
    g = math.gcd(c, groups)
    return nn.GroupNorm(g, c)


class ResBlock(nn.Module):
    """GN-SiLU-conv, + projected time embedding, GN-SiLU-conv, plus a (1x1 if needed) skip."""

    def __init__(self, cin: int, cout: int, temb: int, groups: int = 32):
        super().__init__()
        self.n1, self.c1 = _gn(cin, groups), nn.Conv2d(cin, cout, 3, padding=1)
        self.t = nn.Linear(temb, cout)
        self.n2, self.c2 = _gn(cout, groups), nn.Conv2d(cout, cout, 3, padding=1)
        self.skip = nn.Conv2d(cin, cout, 1) if cin != cout else nn.Identity()

    def forward(self, x, temb):
        h = self.c1(F.silu(self.n1(x)))
        h = h + self.t(F.silu(temb))[:, :, None, None]
        h = self.c2(F.silu(self.n2(h)))
        return self.skip(x) + h


class SpatialTransformer(nn.Module):
    """Tokens = pixels: pre-norm self-attention, optional cross-attention to a context [B, L, ctx],
    GELU feed-forward, with a residual around the whole block."""

    def __init__(self, ch: int, heads: int, context_dim: int | None = None, groups: int = 32):
        super().__init__()
        self.h = heads
        self.norm = _gn(ch, groups)
        self.proj_in, self.proj_out = nn.Conv2d(ch, ch, 1), nn.Conv2d(ch, ch, 1)
        self.ln1, self.qkv, self.o1 = nn.LayerNorm(ch), nn.Linear(ch, 3 * ch, bias=False), nn.Linear(ch, ch)
        self.cross = context_dim is not None
        if self.cross:
            self.ln2, self.q2 = nn.LayerNorm(ch), nn.Linear(ch, ch, bias=False)
            self.kv2, self.o2 = nn.Linear(context_dim, 2 * ch, bias=False), nn.Linear(ch, ch)
        self.ln3 = nn.LayerNorm(ch)
        self.ff = nn.Sequential(nn.Linear(ch, 4 * ch), nn.GELU(), nn.Linear(4 * ch, ch))

    def _heads(self, t):
        B, L, C = t.shape
        return t.view(B, L, self.h, C // self.h).transpose(1, 2)

    def forward(self, x, context=None):
        B, C, H, W = x.shape
        h = self.proj_in(self.norm(x)).flatten(2).transpose(1, 2)  # [B, HW, C]
        q, k, v = self.qkv(self.ln1(h)).chunk(3, -1)
        a = F.scaled_dot_product_attention(self._heads(q), self._heads(k), self._heads(v))
        h = h + self.o1(a.transpose(1, 2).reshape(B, H * W, C))
        if self.cross and context is not None:
            k2, v2 = self.kv2(context).chunk(2, -1)
            a = F.scaled_dot_product_attention(self._heads(self.q2(self.ln2(h))), self._heads(k2), self._heads(v2))
            h = h + self.o2(a.transpose(1, 2).reshape(B, H * W, C))
        h = h + self.ff(self.ln3(h))
        return x + self.proj_out(h.transpose(1, 2).reshape(B, C, H, W))


class Downsample2d(nn.Module):
    def __init__(self, ch: int):
        super().__init__()
        self.conv = nn.Conv2d(ch, ch, 3, stride=2, padding=1)

    def forward(self, x):
        return self.conv(x)


class Upsample2d(nn.Module):
    def __init__(self, ch: int):
        super().__init__()
        self.conv = nn.Conv2d(ch, ch, 3, padding=1)

    def forward(self, x):
        return self.conv(F.interpolate(x, scale_factor=2, mode="nearest"))


class Unet2d(nn.Module):
    """eps_theta(x_t, t, context): x [B, in, H, W] with H, W divisible by 2^(levels - 1)."""

    def __init__(self, config: UnetConfig | None = None):
        super().__init__()
        c = self.config = config or UnetConfig()
        mc, g = c.model_channels, c.groups
        temb = 4 * mc
        self.temb = nn.Sequential(nn.Linear(mc, temb), nn.SiLU(), nn.Linear(temb, temb))
        self.conv_in = nn.Conv2d(c.in_channels, mc, 3, padding=1)
        self.down = nn.ModuleList()
        chans, ch = [mc], mc
        for lvl, mult in enumerate(c.channel_mult):
            for _ in range(c.num_res_blocks):
                blk = nn.ModuleList([ResBlock(ch, mult * mc, temb, g)])
                ch = mult * mc
                if lvl in c.attention_levels:
                    blk.append(SpatialTransformer(ch, c.num_heads, c.context_dim, g))
                self.down.append(blk)
                chans.append(ch)
            if lvl + 1 < len(c.channel_mult):
                self.down.append(nn.ModuleList([Downsample2d(ch)]))
                chans.append(ch)
        self.mid = nn.ModuleList([ResBlock(ch, ch, temb, g), SpatialTransformer(ch, c.num_heads, c.context_dim, g),
                                  ResBlock(ch, ch, temb, g)])
        self.up = nn.ModuleList()
        for lvl, mult in reversed(list(enumerate(c.channel_mult))):
            for i in range(c.num_res_blocks + 1):
                blk = nn.ModuleList([ResBlock(ch + chans.pop(), mult * mc, temb, g)])
                ch = mult * mc
                if lvl in c.attention_levels:
                    blk.append(SpatialTransformer(ch, c.num_heads, c.context_dim, g))
                if lvl > 0 and i == c.num_res_blocks:
                    blk.append(Upsample2d(ch))
                self.up.append(blk)
        self.out = nn.Sequential(_gn(ch, g), nn.SiLU(), nn.Conv2d(ch, c.out_channels, 3, padding=1))

    @staticmethod
    def _run(blk, h, temb, context):
        for m in blk:
            if isinstance(m, ResBlock):
                h = m(h, temb)
            elif isinstance(m, SpatialTransformer):
                h = m(h, context)
            else:
                h = m(h)
        return h

    def forward(self, x, t, context=None):
        t = torch.as_tensor(t, device=x.device)
        if t.dim() == 0:
            t = t.expand(x.shape[0])
        temb = self.temb(timestep_embedding(t, self.config.model_channels).to(x.dtype))
        h = self.conv_in(x)
        skips = [h]
        for blk in self.down:
            h = self._run(blk, h, temb, context)
            skips.append(h)
        h = self._run(self.mid, h, temb, context)
        for blk in self.up:
            h = self._run(blk, torch.cat([h, skips.pop()], 1), temb, context)
        return self.out(h)


# ------------------------------------------------------------------------------------------ sampling
def apply_cfg(uncond_pred: torch.Tensor, cond_pred: torch.Tensor, guidance_scale: float) -> torch.Tensor:
    """Classifier-free guidance: uncond + scale (cond - uncond)."""
    return uncond_pred + guidance_scale * (cond_pred - uncond_pred)


class PlmsSampler:
    """Pseudo linear multistep (PNDM's PLMS): DDIM transfers driven by an Adams-Bashforth combination
    of the last epsilons, (55 e_t - 59 e_{t-1} + 37 e_{t-2} - 9 e_{t-3}) / 24 once four are known; the
    first step uses the second-order pseudo-improved-Euler estimate, then orders 2 and 3 as history
    accumulates."""

    def __init__(self, schedule: NoiseSchedule):
        self.s = schedule

    def _transfer(self, x, eps, ac, ac_prev):
        x0 = (x - math.sqrt(1 - ac) * eps) / math.sqrt(ac)
        return math.sqrt(ac_prev) * x0 + math.sqrt(1 - ac_prev) * eps

    @torch.no_grad()
    def sample(self, model, shape, num_steps: int = 50, device=None, cond=None, guidance_scale: float = 1.0,
               generator=None, x=None, dtype=None):
        T = self.s.timesteps
        ts = torch.linspace(T - 1, 0, num_steps).round().long().tolist()
        if x is None:
            x = torch.randn(shape, generator=generator, device="cpu").to(device=device, dtype=dtype or torch.float32)
        ac_all = self.s.alphas_cumprod
        hist: list[torch.Tensor] = []

        def eps_at(xx, t):
            tt = torch.full((shape[0],), t, dtype=torch.long, device=xx.device)
            return guided_eps(model, xx, tt, cond, guidance_scale)

        for i, t in enumerate(ts):
            ac = float(ac_all[t])
            ac_prev = float(ac_all[ts[i + 1]]) if i + 1 < len(ts) else 1.0
            e = eps_at(x, t)
            if not hist and i + 1 < len(ts):
                # pseudo improved Euler: average the slope here and at the predicted next point
                x_next = self._transfer(x, e, ac, ac_prev)
                e_prime = (e + eps_at(x_next, ts[i + 1])) / 2
            elif len(hist) == 1:
                e_prime = (3 * e - hist[-1]) / 2
            elif len(hist) == 2:
                e_prime = (23 * e - 16 * hist[-1] + 5 * hist[-2]) / 12
            elif len(hist) >= 3:
                e_prime = (55 * e - 59 * hist[-1] + 37 * hist[-2] - 9 * hist[-3]) / 24
            else:
                e_prime = e
            hist.append(e)
            hist = hist[-3:]
            x = self._transfer(x, e_prime, ac, ac_prev)
        return x


# ------------------------------------------------------------------------------------------ conditioning / training
@dataclass
class ConditioningContext:
    """Cross-attention context [B, L, ctx_dim] and an optional null context for guidance."""
    context: torch.Tensor | None = None
    null_context: torch.Tensor | None = None

    def drop(self, p: float, generator=None) -> torch.Tensor | None:
        """Replace each sample's context by the null context with probability p (guidance training)."""
        if self.context is None or p <= 0:
            return self.context
        keep = torch.rand(self.context.shape[0], generator=generator) >= p
        null = self.null_context if self.null_context is not None else torch.zeros_like(self.context[:1])
        return torch.where(keep.to(self.context.device)[:, None, None], self.context, null.expand_as(self.context))


class IdentityLatentCodec:
    """Pixel-space diffusion: encode and decode are the identity (a VAE slots in with the same methods)."""

    def encode(self, x):
        return x

    def decode(self, z):
        return z


class DiffusionTrainer:
    """Epsilon-prediction training of a denoiser ``model(x_t, t, cond)`` with AdamW, gradient clipping
    and an optional EMA copy of the weights for sampling."""

    def __init__(self, model, schedule: NoiseSchedule, lr: float = 2e-4, weight_decay: float = 0.0,
                 grad_clip: float = 1.0, ema_decay: float | None = 0.999):
        self.model, self.s, self.clip = model, schedule, grad_clip
        self.opt = torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=weight_decay)
        self.ema = None
        if ema_decay is not None:
            self.ema_decay = ema_decay
            self.ema = [p.detach().clone() for p in model.parameters()]
        self.steps = 0

    def step(self, x0, cond=None, generator=None) -> float:
        loss = diffusion_loss(self.model, self.s, x0, cond, generator)
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        if self.clip:
            torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.clip)
        self.opt.step()
        if self.ema is not None:
            with torch.no_grad():
                for e, p in zip(self.ema, self.model.parameters()):
                    e.mul_(self.ema_decay).add_(p.detach(), alpha=1 - self.ema_decay)
        self.steps += 1
        return float(loss.detach())
