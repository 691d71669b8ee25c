"""GAN losses, regularisers, StyleGAN-style and CycleGAN-style pieces, evaluation metrics and sampling
utilities, on batched tensors.

Reference: crates/brain-gan/src/losses/classic.rs (relativistic hinge losses), losses/perceptual.rs
(Gram matrix, feature matching, style and perceptual losses), cycle.rs (cycle-consistency and identity
losses, CycleGAN), ops.rs (spectral normalisation by one power iteration, latent interpolation, image
grids, style mixing), stylegan_lite.rs (mapping network, adaptive instance norm, per-layer style
mixing), utils.rs (EMA of weights, weight clipping, LCG Gaussian sampling), eval/ (FID-lite, IS-lite,
fixed latent samples, interpolation sequences, grids), train/penalties.rs (label smoothing).

Differences of form: losses take batches (``[B, ...]`` tensors, averaged over the batch) rather than
one scalar score; the Gram matrix and AdaIN work per channel of ``[B, C, ...]`` feature maps (the
reference's single-vector versions are the B = C = 1 case); the mapping network, StyleGAN synthesis
and CycleGAN generators are trainable modules where the reference keeps zero-weight placeholders.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from ..nn.layers import Linear
from ..nn.module import Module
from ..utils.random import lcg64_unit


# ------------------------------------------------------------------------------------------ losses
def ragan_loss_d(d_real: torch.Tensor, d_fake: torch.Tensor) -> torch.Tensor:
    """Relativistic hinge loss for the discriminator: relu(1 - (r - f)) + relu(1 + (f - r)), batch mean."""
    d_real, d_fake = torch.as_tensor(d_real), torch.as_tensor(d_fake)
    return (F.relu(1.0 - (d_real - d_fake)) + F.relu(1.0 + (d_fake - d_real))).mean()


def ragan_loss_g(d_real: torch.Tensor, d_fake: torch.Tensor) -> torch.Tensor:
    d_real, d_fake = torch.as_tensor(d_real), torch.as_tensor(d_fake)
    return (F.relu(1.0 + (d_real - d_fake)) + F.relu(1.0 - (d_fake - d_real))).mean()


def gram_matrix(features: torch.Tensor) -> torch.Tensor:
    """[B, C, *] -> [B, C, C] channel Gram matrices F F^T (unnormalised); a 1-D vector gives its outer product."""
    if features.dim() == 1:
        return torch.outer(features, features)
    f = features.reshape(features.shape[0], features.shape[1], -1)
    return f @ f.transpose(1, 2)


def feature_matching_loss(real_feats: torch.Tensor, fake_feats: torch.Tensor) -> torch.Tensor:
    """Mean squared difference over the common prefix of the flattened features (0 when empty)."""
    r, f = real_feats.reshape(-1), fake_feats.reshape(-1)
    n = min(r.numel(), f.numel())
    return ((r[:n] - f[:n]) ** 2).mean() if n else r.new_zeros(())


def style_loss(real_feats, fake_feats) -> torch.Tensor:
    return feature_matching_loss(gram_matrix(real_feats), gram_matrix(fake_feats))


@dataclass
class PerceptualConfig:
    feature_weight: float = 10.0
    style_weight: float = 1.0
    num_layers: int = 3


def perceptual_loss(real_feats, fake_feats, config: PerceptualConfig | None = None) -> torch.Tensor:
    """feature_weight * feature matching + style_weight * style loss; lists of per-layer features sum up."""
    c = config or PerceptualConfig()
    if isinstance(real_feats, (list, tuple)):
        return sum(perceptual_loss(r, f, c) for r, f in zip(real_feats[:c.num_layers], fake_feats[:c.num_layers]))
    return c.feature_weight * feature_matching_loss(real_feats, fake_feats) + c.style_weight * style_loss(real_feats,
                                                                                                         fake_feats)


@dataclass
class CycleConfig:
    cycle_lambda: float = 10.0
    identity_lambda: float = 5.0
    latent_dim: int = 64


def cycle_consistency_loss(reconstructed: torch.Tensor, original: torch.Tensor) -> torch.Tensor:
    """Mean absolute difference over the common prefix (L1 cycle loss)."""
    r, o = reconstructed.reshape(-1), original.reshape(-1)
    n = min(r.numel(), o.numel())
    return (r[:n] - o[:n]).abs().mean() if n else r.new_zeros(())


identity_loss = cycle_consistency_loss


def cycle_total_loss(adv_loss, cycle_loss, id_loss, config: CycleConfig | None = None):
    c = config or CycleConfig()
    return adv_loss + c.cycle_lambda * cycle_loss + c.identity_lambda * id_loss


class CycleGan(Module):
    """Two generators A->B and B->A (MLPs over flattened samples, tanh output) with the cycle and
    identity losses of the full CycleGAN objective."""

    def __init__(self, dim: int, hidden: int = 128, config: CycleConfig | None = None, device=None, dtype=None):
        super().__init__()
        self.config = config or CycleConfig()
        self.a2b = torch.nn.Sequential(Linear(dim, hidden, True, device, dtype), torch.nn.ReLU(),
                                       Linear(hidden, dim, True, device, dtype), torch.nn.Tanh())
        self.b2a = torch.nn.Sequential(Linear(dim, hidden, True, device, dtype), torch.nn.ReLU(),
                                       Linear(hidden, dim, True, device, dtype), torch.nn.Tanh())

    def generator_losses(self, real_a, real_b, adv_loss=0.0):
        fake_b, fake_a = self.a2b(real_a), self.b2a(real_b)
        cyc = cycle_consistency_loss(self.b2a(fake_b), real_a) + cycle_consistency_loss(self.a2b(fake_a), real_b)
        idt = identity_loss(self.a2b(real_b), real_b) + identity_loss(self.b2a(real_a), real_a)
        return cycle_total_loss(adv_loss, cyc, idt, self.config), fake_a, fake_b


# ------------------------------------------------------------------------------------------ ops
def spectral_norm_apply(w: torch.Tensor, u: torch.Tensor):
    """One power iteration: v = normalise(W^T u), u' = W v, sigma = u' . u, u' normalised; returns
    (W / sigma, u', sigma) with norms and sigma floored at 1e-8. W is [rows, cols] (trailing dims folded)."""
    w2 = w.reshape(w.shape[0], -1)
    v = w2.t() @ u
    v = v / v.norm().clamp_min(1e-8)
    un = w2 @ v
    sigma = (un * u).sum()
    un = un / un.norm().clamp_min(1e-8)
    s = sigma.clamp_min(1e-8)
    return w / s, un, float(sigma)


def interpolate_latents(a: torch.Tensor, b: torch.Tensor, alpha: float) -> torch.Tensor:
    """alpha a + (1 - alpha) b."""
    return alpha * a + (1.0 - alpha) * b


mix_style = interpolate_latents


def interpolate_latents_batch(z1: torch.Tensor, z2: torch.Tensor, steps: int) -> torch.Tensor:
    """[steps + 1, d]: alpha = s / max(steps, 1) for s = 0..steps, each alpha z1 + (1 - alpha) z2."""
    n = min(z1.numel(), z2.numel())
    alpha = torch.arange(steps + 1, dtype=z1.dtype, device=z1.device)[:, None] / max(steps, 1)
    return alpha * z1.reshape(-1)[:n] + (1.0 - alpha) * z2.reshape(-1)[:n]


def image_grid(images: torch.Tensor, ncols: int, pad: int = 0, value: float = 0.0) -> torch.Tensor:
    """[N, C, H, W] -> [C, rows (H + pad) - pad, ncols (W + pad) - pad], row-major tiling, empty cells = value."""
    n, c, h, w = images.shape
    rows = -(-n // ncols)
    out = images.new_full((c, rows * (h + pad) - pad, ncols * (w + pad) - pad), value)
    for i in range(n):
        r, q = divmod(i, ncols)
        out[:, r * (h + pad):r * (h + pad) + h, q * (w + pad):q * (w + pad) + w] = images[i]
    return out


def adaptive_instance_norm(x: torch.Tensor, style_scale: torch.Tensor, style_bias: torch.Tensor,
                           eps: float = 1e-5) -> torch.Tensor:
    """AdaIN: normalise each (sample, channel) of x [B, C, *] over its spatial positions, then scale and
    shift with per-sample styles [B, C] (a 1-D x is normalised as a whole, the reference's form)."""
    if x.dim() == 1:
        xn = (x - x.mean()) / torch.sqrt(x.var(unbiased=False) + eps)
        k = x.numel()
        return xn * style_scale.reshape(-1).repeat(-(-k // style_scale.numel()))[:k] + \
            style_bias.reshape(-1).repeat(-(-k // style_bias.numel()))[:k]
    dims = tuple(range(2, x.dim()))
    mu = x.mean(dims, keepdim=True)
    var = x.var(dims, unbiased=False, keepdim=True)
    shape = (x.shape[0], x.shape[1]) + (1,) * len(dims)
    return (x - mu) / torch.sqrt(var + eps) * style_scale.reshape(shape) + style_bias.reshape(shape)


def style_mix(w1: torch.Tensor, w2: torch.Tensor, mix_layer: int, num_layers: int) -> list:
    """Per-layer styles: w1 for layers below mix_layer, w2 from there on."""
    return [w1 if l < mix_layer else w2 for l in range(num_layers)]


def track_ema(ema, new_weights, decay: float):
    """decay * ema + (1 - decay) * new, per tensor (in place on the EMA tensors, which are returned)."""
    with torch.no_grad():
        for e, n in zip(ema, new_weights):
            e.mul_(decay).add_(n.detach(), alpha=1.0 - decay)
    return list(ema)


def clip_weights(t: torch.Tensor, clip: float) -> torch.Tensor:
    return t.clamp(-clip, clip)


def smooth_labels(real: float, label_smooth_real: float = 0.9, label_smooth_fake: float = 0.0):
    """One-sided label smoothing: (min(smooth_real, real), smooth_fake)."""
    return min(label_smooth_real, real), label_smooth_fake


def sample_gaussian(dim: int, seed: int) -> torch.Tensor:
    """dim normals from the LCG stream seeded with ``seed``: per value u1 = max(draw, 1e-15), u2 = draw,
    sqrt(-2 ln u1) cos(2 pi u2)."""
    u = lcg64_unit(seed, 2 * dim)
    u1, u2 = np.maximum(u[0::2], 1e-15), u[1::2]
    return torch.from_numpy(np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * math.pi * u2))


def fixed_latent_sample(latent_dim: int, n: int, seed: int) -> torch.Tensor:
    """[n, latent_dim]: row i is sample_gaussian(latent_dim, seed + i 0xdeadbeef)."""
    return torch.stack([sample_gaussian(latent_dim, (seed + i * 0xDEADBEEF) & ((1 << 64) - 1)) for i in range(n)])


# ------------------------------------------------------------------------------------------ evaluation
def fid_lite(real_feats: torch.Tensor, fake_feats: torch.Tensor) -> float:
    """Squared distance between the feature means ([N, d] each; the covariance term of FID is left out)."""
    if real_feats.numel() == 0 or fake_feats.numel() == 0:
        return 0.0
    r = real_feats.double().reshape(real_feats.shape[0], -1).mean(0)
    f = fake_feats.double().reshape(fake_feats.shape[0], -1).mean(0)
    return float(((r - f) ** 2).sum())


def is_lite(logits: torch.Tensor) -> float:
    """exp(mean entropy of softmax(logits) / ln(classes)) over the rows of [N, classes]; 1 when empty."""
    if logits.numel() == 0:
        return 1.0
    lg = logits.double().reshape(logits.shape[0], -1)
    p = torch.softmax(lg, 1)
    h = -(p * p.clamp_min(1e-15).log()).sum(1).mean()
    return float(torch.exp(h / max(math.log(lg.shape[1]), 1e-8)))


@dataclass
class GanEvalReport:
    fid_lite: float = 0.0
    is_lite: float = 0.0
    avg_d_real: float = 0.0
    avg_d_fake: float = 0.0
    num_samples: int = 0

    def summary(self) -> str:
        return (f"EvalReport[FID-lite={self.fid_lite:.4f} IS-lite={self.is_lite:.4f} D(real)={self.avg_d_real:.4f} "
                f"D(fake)={self.avg_d_fake:.4f} n={self.num_samples}]")


def eval_gan(real: torch.Tensor, fake: torch.Tensor, d_real=None, d_fake=None) -> GanEvalReport:
    """FID-lite between real and fake, IS-lite of fake, and the mean discriminator outputs when given
    (else tanh of each sample's sum, the reference's stand-in)."""
    dr = d_real if d_real is not None else torch.tanh(real.double().reshape(real.shape[0], -1).sum(1))
    df = d_fake if d_fake is not None else torch.tanh(fake.double().reshape(fake.shape[0], -1).sum(1))
    return GanEvalReport(fid_lite(real, fake), is_lite(fake), float(dr.mean()), float(df.mean()), int(fake.shape[0]))


# ------------------------------------------------------------------------------------------ StyleGAN-style
class MappingNetwork(Module):
    """z -> w: ``num_layers`` linear layers with LeakyReLU(0.2); weights stored at unit scale and
    multiplied by lr_multiplier / sqrt(fan_in) in the forward pass (equalised learning rate)."""

    def __init__(self, latent_dim: int = 512, style_dim: int = 512, num_layers: int = 8, lr_multiplier: float = 0.01,
                 device=None, dtype=None):
        super().__init__()
        self.lrm = lr_multiplier
        dims = [latent_dim] + [style_dim] * num_layers
        self.weights = torch.nn.ParameterList(
            [torch.nn.Parameter(torch.randn(dims[i + 1], dims[i], device=device, dtype=dtype) / lr_multiplier)
             for i in range(num_layers)])
        self.biases = torch.nn.ParameterList(
            [torch.nn.Parameter(torch.zeros(dims[i + 1], device=device, dtype=dtype)) for i in range(num_layers)])

    def forward(self, z: torch.Tensor) -> torch.Tensor:
        x = z * torch.rsqrt((z * z).mean(-1, keepdim=True) + 1e-8)  # pixel norm of the latent
        for w, b in zip(self.weights, self.biases):
            x = F.leaky_relu(F.linear(x, w * (self.lrm / math.sqrt(w.shape[1])), b * self.lrm), 0.2)
        return x


class StyleGanLite(Module):
    """Mapping network plus a synthesis stack: a learned 4x4 constant, then per layer a 2x nearest
    upsample (every other layer), a 3x3 convolution, noise-free AdaIN from an affine map of w, and
    LeakyReLU; a 1x1 conv to RGB. ``forward(z)`` or ``synthesize(list of per-layer w)`` for mixing."""

    def __init__(self, latent_dim: int = 64, style_dim: int = 64, output_size: int = 16, channels: int = 32,
                 mapping_layers: int = 4, device=None, dtype=None):
        super().__init__()
        self.mapping = MappingNetwork(latent_dim, style_dim, mapping_layers, 0.01, device, dtype)
        ups = int(round(math.log2(output_size / 4)))
        self.num_layers = 2 * ups + 1
        self.const = torch.nn.Parameter(torch.randn(1, channels, 4, 4, device=device, dtype=dtype))
        self.convs = torch.nn.ModuleList(
            torch.nn.Conv2d(channels, channels, 3, padding=1, device=device, dtype=dtype) for _ in range(self.num_layers))
        self.affine = torch.nn.ModuleList(
            Linear(style_dim, 2 * channels, True, device, dtype) for _ in range(self.num_layers))
        self.to_rgb = torch.nn.Conv2d(channels, 3, 1, device=device, dtype=dtype)

    def synthesize(self, ws) -> torch.Tensor:
        x = self.const.expand(ws[0].shape[0], -1, -1, -1)
        for l, (conv, aff) in enumerate(zip(self.convs, self.affine)):
            if l % 2 == 1:
                x = F.interpolate(x, scale_factor=2, mode="nearest")
            st = aff(ws[l])
            scale, bias = st.chunk(2, -1)
            x = F.leaky_relu(adaptive_instance_norm(conv(x), 1.0 + scale, bias), 0.2)
        return torch.tanh(self.to_rgb(x))

    def forward(self, z: torch.Tensor) -> torch.Tensor:
        w = self.mapping(z)
        return self.synthesize([w] * self.num_layers)


# ------------------------------------------------------------------------------------------ more architectures
# Reference: discriminator/patch.rs (PatchDiscriminator, num_patches), generator/resnet.rs
# (ResnetGenerator: residual blocks between down- and up-sampling), generator/conditional.rs
# (class embedding concatenated to z), discriminator/conditional.rs (class projection added to the
# score), train/mod.rs + train/loop_.rs (GanTrainer, n_critic, per-epoch statistics), eval/samples.rs
# (assemble_grid).

def _norm2d(kind: str, c: int, device=None, dtype=None):
    if kind == "batch":
        return torch.nn.BatchNorm2d(c, device=device, dtype=dtype)
    if kind == "instance":
        return torch.nn.InstanceNorm2d(c, affine=True, device=device, dtype=dtype)
    return torch.nn.Identity()


class PatchDiscriminator(Module):
    """PatchGAN: 4x4 stride-2 convs (LeakyReLU 0.2, normalised after the first) then a stride-1 conv to
    one logit per receptive-field patch: [B, 1, h, w]."""

    def __init__(self, in_channels: int = 3, base: int = 64, n_layers: int = 3, norm: str = "batch", device=None,
                 dtype=None):
        super().__init__()
        layers, c = [], in_channels
        for i in range(n_layers):
            co = base * 2 ** i
            layers.append(torch.nn.Conv2d(c, co, 4, 2, 1, device=device, dtype=dtype))
            if i > 0:
                layers.append(_norm2d(norm, co, device, dtype))
            layers.append(torch.nn.LeakyReLU(0.2))
            c = co
        layers.append(torch.nn.Conv2d(c, 1, 3, 1, 1, device=device, dtype=dtype))
        self.net = torch.nn.Sequential(*layers)
        self.n_layers = n_layers

    def num_patches(self, h: int, w: int) -> int:
        return (h >> self.n_layers) * (w >> self.n_layers)

    def forward(self, x):
        return self.net(x)


class _ResBlock(Module):
    def __init__(self, c, norm, device=None, dtype=None):
        super().__init__()
        self.body = torch.nn.Sequential(
            torch.nn.ReflectionPad2d(1), torch.nn.Conv2d(c, c, 3, device=device, dtype=dtype), _norm2d(norm, c, device, dtype),
            torch.nn.ReLU(), torch.nn.ReflectionPad2d(1), torch.nn.Conv2d(c, c, 3, device=device, dtype=dtype),
            _norm2d(norm, c, device, dtype))

    def forward(self, x):
        return x + self.body(x)


class ResnetGenerator(Module):
    """Image-to-image generator: 7x7 stem, two stride-2 down-samplings, ``n_blocks`` residual blocks,
    two stride-2 transposed-conv up-samplings, 7x7 head with tanh. Output has the input's H x W."""

    def __init__(self, in_channels: int = 3, out_channels: int = 3, base: int = 64, n_blocks: int = 6,
                 norm: str = "batch", device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        layers = [torch.nn.ReflectionPad2d(3), torch.nn.Conv2d(in_channels, base, 7, **kw), _norm2d(norm, base, **kw),
                  torch.nn.ReLU()]
        c = base
        for _ in range(2):
            layers += [torch.nn.Conv2d(c, 2 * c, 3, 2, 1, **kw), _norm2d(norm, 2 * c, **kw), torch.nn.ReLU()]
            c *= 2
        layers += [_ResBlock(c, norm, **kw) for _ in range(n_blocks)]
        for _ in range(2):
            layers += [torch.nn.ConvTranspose2d(c, c // 2, 3, 2, 1, output_padding=1, **kw), _norm2d(norm, c // 2, **kw),
                       torch.nn.ReLU()]
            c //= 2
        layers += [torch.nn.ReflectionPad2d(3), torch.nn.Conv2d(c, out_channels, 7, **kw), torch.nn.Tanh()]
        self.net = torch.nn.Sequential(*layers)

    def forward(self, x):
        return self.net(x)


class ConditionalGenerator(Module):
    """G(z, y): a learned class embedding of size latent_dim is concatenated to z and fed to an MLP
    generator producing ``out_dim`` values in (-1, 1)."""

    def __init__(self, latent_dim: int, num_classes: int, out_dim: int, hidden: int = 256, device=None, dtype=None):
        super().__init__()
        self.latent_dim, self.num_classes = latent_dim, num_classes
        self.embed = torch.nn.Embedding(num_classes, latent_dim, device=device, dtype=dtype)
        self.net = torch.nn.Sequential(Linear(2 * latent_dim, hidden, True, device, dtype), torch.nn.ReLU(),
                                       Linear(hidden, hidden, True, device, dtype), torch.nn.ReLU(),
                                       Linear(hidden, out_dim, True, device, dtype), torch.nn.Tanh())

    def embed_class(self, y):
        return self.embed(torch.as_tensor(y, device=self.embed.weight.device).long())

    def forward(self, z, y):
        return self.net(torch.cat([z, self.embed_class(y)], -1))


class ConditionalDiscriminator(Module):
    """Projection discriminator (Miyato & Koyama 2018): D(x, y) = w . phi(x) + <e_y, phi(x)>."""

    def __init__(self, in_dim: int, num_classes: int, hidden: int = 256, device=None, dtype=None):
        super().__init__()
        self.phi = torch.nn.Sequential(Linear(in_dim, hidden, True, device, dtype), torch.nn.LeakyReLU(0.2),
                                       Linear(hidden, hidden, True, device, dtype), torch.nn.LeakyReLU(0.2))
        self.out = Linear(hidden, 1, True, device, dtype)
        self.class_embed = torch.nn.Embedding(num_classes, hidden, device=device, dtype=dtype)

    def class_projection(self, features, y):
        e = self.class_embed(torch.as_tensor(y, device=features.device).long())
        return (e * features).sum(-1, keepdim=True)

    def forward(self, x, y):
        h = self.phi(x)
        return self.out(h) + self.class_projection(h, y)


@dataclass
class GanTrainStats:
    epoch: int
    d_loss: float
    g_loss: float
    steps: int


class GanTrainer:
    """Alternating updates over a data iterable: ``n_critic`` discriminator steps per generator step,
    an optional gradient penalty, per-epoch mean losses. ``loss`` is one of bce / hinge / lsgan / wgan."""

    def __init__(self, gen, disc, opt_g, opt_d, loss: str = "bce", n_critic: int = 1, gp_weight: float = 0.0,
                 clip: float | None = None, seed: int = 0):
        from .gan import (bce_loss_d, bce_loss_g, gradient_penalty, hinge_loss_d, hinge_loss_g, lsgan_loss_d,
                          lsgan_loss_g, wgan_loss_d, wgan_loss_g)
        self.gen, self.disc, self.opt_g, self.opt_d = gen, disc, opt_g, opt_d
        self.ld = {"bce": bce_loss_d, "hinge": hinge_loss_d, "lsgan": lsgan_loss_d, "wgan": wgan_loss_d}[loss]
        self.lg = {"bce": bce_loss_g, "hinge": hinge_loss_g, "lsgan": lsgan_loss_g, "wgan": wgan_loss_g}[loss]
        self.gp, self.gp_weight, self.n_critic, self.clip = gradient_penalty, gp_weight, n_critic, clip
        self.g = torch.Generator().manual_seed(seed)
        self.history: list[GanTrainStats] = []

    def _z(self, n, ref):
        return torch.randn((n, self.gen.latent_dim), generator=self.g).to(ref.device, ref.dtype)

    def discriminator_step(self, real) -> float:
        fake = self.gen(self._z(real.shape[0], real)).detach()
        ld = self.ld(self.disc(real), self.disc(fake))
        if self.gp_weight > 0:
            ld = ld + self.gp(self.disc, real, fake, self.gp_weight, self.g)
        self.opt_d.zero_grad()
        ld.backward()
        self.opt_d.step()
        if self.clip is not None:  # WGAN weight clipping
            with torch.no_grad():
                for prm in self.disc.parameters():
                    prm.copy_(clip_weights(prm, self.clip))
        return float(ld.detach())

    def generator_step(self, batch_size: int, ref) -> float:
        lg = self.lg(self.disc(self.gen(self._z(batch_size, ref))))
        self.opt_g.zero_grad()
        lg.backward()
        self.opt_g.step()
        return float(lg.detach())

    def train_epoch(self, data) -> GanTrainStats:
        dl, gl, nd, ng = 0.0, 0.0, 0, 0
        for i, real in enumerate(data):
            dl += self.discriminator_step(real)
            nd += 1
            if (i + 1) % self.n_critic == 0:
                gl += self.generator_step(real.shape[0], real)
                ng += 1
        st = GanTrainStats(len(self.history), dl / max(nd, 1), gl / max(ng, 1), nd)
        self.history.append(st)
        return st

    def fit(self, data_fn, epochs: int) -> list[GanTrainStats]:
        return [self.train_epoch(data_fn()) for _ in range(epochs)]


def assemble_grid(images: torch.Tensor, ncols: int, pad: int = 2, value: float = 1.0) -> torch.Tensor:
    return image_grid(images, ncols, pad, value)
