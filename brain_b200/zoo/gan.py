"""Generative adversarial networks: adversarial losses (BCE, hinge, least squares, WGAN), gradient
penalties (WGAN-GP, R1, R2), label smoothing, MLP and DCGAN-style generator / discriminator, and a
training step.

Reference: crates/brain-gan. Losses (losses/classic.rs:10-100: hinge, WGAN, WGAN-GP with interpolates,
R1/R2, LSGAN, BCE with label smoothing), penalties (train/penalties.rs:10-80), generators and
discriminators (generator/dcgan.rs, discriminator/dcgan.rs, discriminator/patch.rs), training loop
(train/loop_.rs).

The reference evaluates penalties on scalar scores it is handed; here they are computed with autograd
(the gradient of D at the interpolates / real samples), which is the quantity the formulas define.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..nn.layers import Linear
from ..nn.module import Module


def bce_loss_d(d_real, d_fake, label_smooth: float = 0.0):
    return (F.binary_cross_entropy_with_logits(d_real, torch.full_like(d_real, 1.0 - label_smooth)) +
            F.binary_cross_entropy_with_logits(d_fake, torch.zeros_like(d_fake)))


def bce_loss_g(d_fake):
    return F.binary_cross_entropy_with_logits(d_fake, torch.ones_like(d_fake))


def hinge_loss_d(d_real, d_fake):
    return F.relu(1 - d_real).mean() + F.relu(1 + d_fake).mean()


def hinge_loss_g(d_fake):
    return -d_fake.mean()


def lsgan_loss_d(d_real, d_fake):
    return 0.5 * ((d_real - 1) ** 2).mean() + 0.5 * (d_fake ** 2).mean()


def lsgan_loss_g(d_fake):
    return 0.5 * ((d_fake - 1) ** 2).mean()


def wgan_loss_d(d_real, d_fake):
    return d_fake.mean() - d_real.mean()


def wgan_loss_g(d_fake):
    return -d_fake.mean()


def sample_wgan_gp_interpolates(real, fake, generator=None):
    eps = torch.rand((real.shape[0],) + (1,) * (real.dim() - 1), generator=generator, device="cpu")
    eps = eps.to(real.device, real.dtype)
    return (eps * real + (1 - eps) * fake).requires_grad_(True)


def _grad_norm_sq(disc, x):
    x = x if x.requires_grad else x.detach().requires_grad_(True)
    out = disc(x)
    (g,) = torch.autograd.grad(out.sum(), x, create_graph=True)
    return g.reshape(g.shape[0], -1).pow(2).sum(1)


def gradient_penalty(disc, real, fake, lam: float = 10.0, generator=None):
    """WGAN-GP: λ E[(‖∇D(x̂)‖ − 1)²] at random interpolates x̂."""
    xi = sample_wgan_gp_interpolates(real.detach(), fake.detach(), generator)
    return lam * ((_grad_norm_sq(disc, xi).sqrt() - 1) ** 2).mean()


def r1_penalty(disc, real, gamma: float = 10.0):
    """R1: (γ / 2) E[‖∇D(x_real)‖²]."""
    return 0.5 * gamma * _grad_norm_sq(disc, real.detach()).mean()


def r2_penalty(disc, fake, gamma: float = 10.0):
    return 0.5 * gamma * _grad_norm_sq(disc, fake.detach()).mean()


class MlpGenerator(Module):
    def __init__(self, latent_dim: int, out_dim: int, hidden: int = 128, device=None, dtype=None):
        super().__init__()
        self.latent_dim = latent_dim
        self.l1 = Linear(latent_dim, hidden, True, device, dtype)
        self.l2 = Linear(hidden, hidden, True, device, dtype)
        self.l3 = Linear(hidden, out_dim, True, device, dtype)

    def forward(self, z):
        return self.l3(F.leaky_relu(self.l2(F.leaky_relu(self.l1(z), 0.2)), 0.2))


class MlpDiscriminator(Module):
    def __init__(self, in_dim: int, hidden: int = 128, device=None, dtype=None):
        super().__init__()
        self.l1 = Linear(in_dim, hidden, True, device, dtype)
        self.l2 = Linear(hidden, hidden, True, device, dtype)
        self.l3 = Linear(hidden, 1, True, device, dtype)

    def forward(self, x):
        return self.l3(F.leaky_relu(self.l2(F.leaky_relu(self.l1(x), 0.2)), 0.2)).squeeze(-1)


class DcganGenerator(Module):
    """z -> 4x4 feature map -> transposed-conv upsampling x2 per stage -> tanh image."""

    def __init__(self, latent_dim: int = 64, channels: int = 1, base: int = 64, stages: int = 3, device=None,
                 dtype=None):
        super().__init__()
        self.base, self.latent_dim = base, latent_dim
        c = base * 2 ** (stages - 1)
        self.proj = Linear(latent_dim, c * 16, True, device, dtype)
        layers = []
        for s in range(stages):
            co = channels if s == stages - 1 else c // 2
            layers.append(torch.nn.ConvTranspose2d(c, co, 4, 2, 1, device=device, dtype=dtype))
            if s < stages - 1:
                layers += [torch.nn.BatchNorm2d(co, device=device, dtype=dtype), torch.nn.ReLU()]
            c = co
        self.net = torch.nn.Sequential(*layers)
        self.c0 = base * 2 ** (stages - 1)

    def forward(self, z):
        return torch.tanh(self.net(F.relu(self.proj(z)).view(z.shape[0], self.c0, 4, 4)))


class DcganDiscriminator(Module):
    """Strided convs (LeakyReLU 0.2) -> one logit; ``patch=True`` keeps the last feature map as a grid
    of per-patch logits (PatchGAN)."""

    def __init__(self, channels: int = 1, base: int = 64, stages: int = 3, patch: bool = False, device=None,
                 dtype=None):
        super().__init__()
        layers, c = [], channels
        for s in range(stages):
            layers += [torch.nn.Conv2d(c, base * 2 ** s, 4, 2, 1, device=device, dtype=dtype),
                       torch.nn.LeakyReLU(0.2)]
            c = base * 2 ** s
        self.net = torch.nn.Sequential(*layers)
        self.out = torch.nn.Conv2d(c, 1, 3 if patch else 4, 1, 1 if patch else 0, device=device, dtype=dtype)
        self.patch = patch

    def forward(self, x):
        y = self.out(self.net(x))
        return y.flatten(1) if self.patch else y.flatten(1).mean(1)


def train_step(gen, disc, opt_g, opt_d, real, loss: str = "bce", gp: float = 0.0, generator=None):
    """One discriminator and one generator update; returns (d_loss, g_loss) as floats."""
    z = torch.randn((real.shape[0], gen.latent_dim), generator=generator, device="cpu").to(real.device, real.dtype)
    fake = gen(z)
    d_real, d_fake = disc(real), disc(fake.detach())
    ld = {"bce": bce_loss_d, "hinge": hinge_loss_d, "lsgan": lsgan_loss_d, "wgan": wgan_loss_d}[loss](d_real, d_fake)
    if gp > 0:
        ld = ld + gradient_penalty(disc, real, fake, gp, generator)
    opt_d.zero_grad()
    ld.backward()
    opt_d.step()
    lg = {"bce": bce_loss_g, "hinge": hinge_loss_g, "lsgan": lsgan_loss_g, "wgan": wgan_loss_g}[loss](disc(fake))
    opt_g.zero_grad()
    lg.backward()
    opt_g.step()
    return float(ld.detach()), float(lg.detach())
