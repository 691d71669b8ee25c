"""ViT utilities: position-embedding construction and resolution change, patch/token operators, masked
token selection, stochastic depth, attention rollout and entropy, a DINO projection head, the NT-Xent
contrastive loss, and a model card.

Reference: crates/brain-vit/src/patch/pos_embed.rs (sinusoidal 1-D / 2-D tables, interpolate_to with a
class token), utils.rs (interpolate_2d, attention_rollout, attention_entropy, nt_xent_loss), ops.rs
(patchify / unpatchify, add / split class token, mask_patches, stochastic_depth_scale,
token_interpolate), vit/heads.rs (DinoHead), export/mod.rs (ModelCard).

The resolution change resamples all embedding channels at once (bilinear on an align-corners grid,
the reference's mapping) as one gather-and-blend over the [D, h, w] table; rollout multiplies the
per-layer [B, N, N] maps on the device; the contrastive loss is one [2B, 2B] similarity GEMM.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from ..nn.layers import Linear
from ..nn.module import Module


# ------------------------------------------------------------------------------------------ position embeddings
def sinusoidal_1d(seq_len: int, dim: int) -> torch.Tensor:
    """[seq_len, dim]: sin at even channels, cos at odd ones, angle pos / 10000^(2 floor(i/2) / dim)."""
    pos = torch.arange(seq_len, dtype=torch.float64)[:, None]
    i = torch.arange(dim)
    ang = pos / (10000.0 ** (2.0 * (i // 2).double() / dim))[None, :]
    return torch.where((i % 2 == 0)[None, :], torch.sin(ang), torch.cos(ang))


def sinusoidal_2d(grid_h: int, grid_w: int, dim: int) -> torch.Tensor:
    """[h w, dim] row-major over the grid: channel 2i = sin(y omega_i), channel 2i + 1 = cos(x omega_i),
    omega_i = 10000^(-2i / dim) (the reference's layout)."""
    ys, xs = torch.meshgrid(torch.arange(grid_h, dtype=torch.float64), torch.arange(grid_w, dtype=torch.float64),
                            indexing="ij")
    om = 1.0 / 10000.0 ** (2.0 * torch.arange(dim // 2, dtype=torch.float64) / dim)
    out = torch.zeros(grid_h * grid_w, dim, dtype=torch.float64)
    out[:, 0:2 * (dim // 2):2] = torch.sin(ys.reshape(-1, 1) * om)
    out[:, 1:2 * (dim // 2):2] = torch.cos(xs.reshape(-1, 1) * om)
    return out


def interpolate_2d(grid: torch.Tensor, new_h: int, new_w: int) -> torch.Tensor:
    """Bilinear resampling of [..., h, w] with corners aligned (source position n (h-1)/(new-1))."""
    h, w = grid.shape[-2:]
    if new_h <= 0 or new_w <= 0:
        raise ValueError("new dimensions must be > 0")
    fy = torch.arange(new_h, dtype=torch.float64) * (h - 1) / max(new_h - 1, 1)
    fx = torch.arange(new_w, dtype=torch.float64) * (w - 1) / max(new_w - 1, 1)
    y0, x0 = fy.floor().long(), fx.floor().long()
    y1, x1 = (y0 + 1).clamp(max=h - 1), (x0 + 1).clamp(max=w - 1)
    ty, tx = (fy - y0)[:, None].to(grid), (fx - x0)[None, :].to(grid)
    g = grid
    v00, v01 = g[..., y0[:, None], x0[None, :]], g[..., y0[:, None], x1[None, :]]
    v10, v11 = g[..., y1[:, None], x0[None, :]], g[..., y1[:, None], x1[None, :]]
    return v00 * (1 - ty) * (1 - tx) + v01 * (1 - ty) * tx + v10 * ty * (1 - tx) + v11 * ty * tx


def interpolate_pos_embed(pos: torch.Tensor, old_hw, new_hw, has_cls: bool = True) -> torch.Tensor:
    """[1 (or none), cls + old_h old_w, D] -> the same for a new patch grid; the class row is kept."""
    squeeze = pos.dim() == 2
    p = pos[None] if squeeze else pos
    (oh, ow), (nh, nw) = old_hw, new_hw
    cls, grid = (p[:, :1], p[:, 1:]) if has_cls else (p[:, :0], p)
    g = grid.reshape(p.shape[0], oh, ow, -1).permute(0, 3, 1, 2)  # [1, D, h, w]
    g = interpolate_2d(g, nh, nw).permute(0, 2, 3, 1).reshape(p.shape[0], nh * nw, -1)
    out = torch.cat([cls, g], 1)
    return out[0] if squeeze else out


# ------------------------------------------------------------------------------------------ tokens
def patchify(images: torch.Tensor, patch: int) -> torch.Tensor:
    """[B, C, H, W] -> [B, (H/p)(W/p), C p p] in row-major patch order, channels outermost within a patch."""
    B, C, H, W = images.shape
    x = images.reshape(B, C, H // patch, patch, W // patch, patch).permute(0, 2, 4, 1, 3, 5)
    return x.reshape(B, (H // patch) * (W // patch), C * patch * patch)


def unpatchify(tokens: torch.Tensor, patch: int, channels: int, h: int, w: int) -> torch.Tensor:
    """Inverse of patchify for an image of h x w pixels."""
    B = tokens.shape[0]
    x = tokens.reshape(B, h // patch, w // patch, channels, patch, patch).permute(0, 3, 1, 4, 2, 5)
    return x.reshape(B, channels, h, w)


def add_cls_token(tokens: torch.Tensor, cls: torch.Tensor) -> torch.Tensor:
    return torch.cat([cls.reshape(1, 1, -1).expand(tokens.shape[0], -1, -1), tokens], 1)


def split_cls_token(tokens: torch.Tensor):
    return tokens[:, 0], tokens[:, 1:]


def mask_patches(tokens: torch.Tensor, keep_mask: torch.Tensor):
    """Keep the tokens whose mask entry is True, in order: [B, N, D] -> ([B, kept, D], kept indices)."""
    idx = keep_mask.nonzero().reshape(-1)
    return tokens[:, idx], idx


def random_keep_mask(num_tokens: int, mask_ratio: float, generator=None) -> torch.Tensor:
    """MAE-style: keep round(N (1 - ratio)) randomly chosen tokens."""
    keep = int(round(num_tokens * (1.0 - mask_ratio)))
    perm = torch.randperm(num_tokens, generator=generator)
    m = torch.zeros(num_tokens, dtype=torch.bool)
    m[perm[:keep]] = True
    return m


def stochastic_depth_scale(rate: float, training: bool, batch: int = 1, generator=None) -> torch.Tensor:
    """Per-sample residual-branch scale: 0 with probability rate, else 1 / (1 - rate); 1 in eval."""
    if not training or rate <= 0:
        return torch.ones(batch)
    keep = (torch.rand(batch, generator=generator) >= rate).double()
    return keep / (1.0 - rate)


# ------------------------------------------------------------------------------------------ analysis
def attention_rollout(attns: torch.Tensor) -> torch.Tensor:
    """attns [L, (B,) N, N] (head-averaged) -> prod over layers of (0.5 A + 0.5 I), last layer leftmost."""
    n = attns.shape[-1]
    eye = torch.eye(n, dtype=attns.dtype, device=attns.device)
    out = eye.expand_as(attns[0]).clone()
    for a in attns:
        out = (0.5 * a + 0.5 * eye) @ out
    return out


def attention_entropy(attn: torch.Tensor) -> torch.Tensor:
    """Row entropies (nats) of attention maps [..., N, N], ignoring probabilities <= 1e-12."""
    p = attn.double()
    return -torch.where(p > 1e-12, p * p.clamp_min(1e-300).log(), torch.zeros_like(p)).sum(-1)


def nt_xent_loss(z1: torch.Tensor, z2: torch.Tensor, temperature: float = 0.5) -> torch.Tensor:
    """SimCLR NT-Xent: over the 2B embeddings, each one's positive is its other view, negatives are all
    other embeddings (itself excluded); similarities are raw dot products / temperature, as in the
    reference (normalise the embeddings first for cosine similarities). Mean over the 2B anchors."""
    z = torch.cat([z1, z2], 0)
    n, b = z.shape[0], z1.shape[0]
    sim = (z @ z.t()) / temperature
    sim = sim.masked_fill(torch.eye(n, dtype=torch.bool, device=z.device), float("-inf"))
    pos = torch.cat([torch.arange(b, n), torch.arange(0, b)]).to(z.device)
    return F.cross_entropy(sim, pos)


# ------------------------------------------------------------------------------------------ heads / export
class DinoHead(Module):
    """DINO projection: Linear-GELU(tanh)-Linear-GELU(tanh)-Linear(no bias), rows L2-normalised."""

    def __init__(self, embed_dim: int, hidden_dim: int = 2048, proj_dim: int = 256, device=None, dtype=None):
        super().__init__()
        if min(embed_dim, hidden_dim, proj_dim) <= 0:
            raise ValueError("DinoHead: all dims must be > 0")
        self.l1 = Linear(embed_dim, hidden_dim, True, device, dtype)
        self.l2 = Linear(hidden_dim, hidden_dim, True, device, dtype)
        self.l3 = Linear(hidden_dim, proj_dim, False, device, dtype)

    def forward(self, pooled: torch.Tensor) -> torch.Tensor:
        h = F.gelu(self.l1(pooled), approximate="tanh")
        h = F.gelu(self.l2(h), approximate="tanh")
        return F.normalize(self.l3(h), dim=-1, eps=1e-12)


@dataclass
class ModelCard:
    name: str
    architecture: str
    num_params: int
    config: dict = field(default_factory=dict)
    metrics: dict = field(default_factory=dict)

    @classmethod
    def for_model(cls, name: str, model, config=None) -> "ModelCard":
        cfg = config if isinstance(config, dict) else (vars(config) if config is not None else {})
        return cls(name, type(model).__name__, sum(p.numel() for p in model.parameters()), dict(cfg))

    def add_metric(self, key: str, value: float) -> None:
        self.metrics[key] = float(value)

    def to_markdown(self) -> str:
        lines = [f"# {self.name}", "", f"- architecture: {self.architecture}", f"- parameters: {self.num_params:,}"]
        if self.config:
            lines += ["", "## Configuration", ""] + [f"- {k}: {v}" for k, v in sorted(self.config.items())]
        if self.metrics:
            lines += ["", "## Metrics", "", "| metric | value |", "|---|---|"] + \
                     [f"| {k} | {v:.4f} |" for k, v in sorted(self.metrics.items())]
        return "\n".join(lines) + "\n"


# ------------------------------------------------------------------ the reference's ViT entry points
# crates/brain-vit/src: patch/mod.rs (PatchEmbed, num_patches_for), impl.rs (VitModel, embed_patches,
# forward_features), vit/heads.rs (VitHead: class-token or mean pooling -> linear), training/mod.rs
# (label_smooth_ce, GradientClipper), ops.rs (position_ids, reconstruct_patches).

def num_patches_for(image_size: int, patch_size: int) -> int:
    if image_size % patch_size:
        raise ValueError(f"image size {image_size} is not a multiple of patch size {patch_size}")
    return (image_size // patch_size) ** 2


class PatchEmbed(torch.nn.Module):
    """Non-overlapping P x P patches -> D features: a reshape then one GEMM (the framework's Linear),
    the same product as a stride-P convolution without an im2col pass."""

    def __init__(self, in_channels: int, patch_size: int, dim: int, device=None, dtype=None):
        super().__init__()
        from ..nn.layers import Linear
        self.P = patch_size
        self.proj = Linear(in_channels * patch_size * patch_size, dim, True, device, dtype)

    def forward(self, images):
        B, C, H, W = images.shape
        P = self.P
        x = images.reshape(B, C, H // P, P, W // P, P).permute(0, 2, 4, 1, 3, 5).reshape(B, -1, C * P * P)
        return self.proj(x.to(self.proj.weight.dtype))


class VitHead(torch.nn.Module):
    """Pooling ("cls": the class token, "mean": mean of the patch tokens) -> LayerNorm -> Linear."""

    def __init__(self, dim: int, num_classes: int, pool: str = "cls", device=None, dtype=None):
        super().__init__()
        from ..nn.layers import Linear
        self.pool = pool
        self.norm = torch.nn.LayerNorm(dim, device=device, dtype=dtype)
        self.fc = Linear(dim, num_classes, True, device, dtype)

    def forward(self, tokens):
        x = tokens[:, 0] if self.pool == "cls" else tokens[:, 1:].mean(1)
        return self.fc(self.norm(x))


def position_ids(num_tokens: int, batch: int = 1, device=None) -> torch.Tensor:
    return torch.arange(num_tokens, device=device).expand(batch, num_tokens)


def reconstruct_patches(patches: torch.Tensor, image_size: int, patch_size: int, channels: int) -> torch.Tensor:
    """[B, N, C*P*P] -> [B, C, H, W] (inverse of patchify)."""
    g = image_size // patch_size
    B = patches.shape[0]
    x = patches.reshape(B, g, g, channels, patch_size, patch_size).permute(0, 3, 1, 4, 2, 5)
    return x.reshape(B, channels, image_size, image_size)


def label_smooth_ce(logits: torch.Tensor, labels: torch.Tensor, smoothing: float = 0.1) -> torch.Tensor:
    return torch.nn.functional.cross_entropy(logits.float(), labels, label_smoothing=smoothing)


class GradientClipper:
    """Global-norm clipping of a parameter set; ``clip`` returns the norm before clipping."""

    def __init__(self, max_norm: float = 1.0):
        self.max_norm = max_norm

    def clip(self, params) -> float:
        return float(torch.nn.utils.clip_grad_norm_(list(params), self.max_norm))
