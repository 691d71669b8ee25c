"""Denoising diffusion: noise schedules, the forward process, the epsilon-prediction loss, DDPM and
DDIM samplers, classifier-free guidance, and a small time-conditioned denoiser.

Reference: crates/brain-diffusion. Schedules (schedules/linear.rs:9-40, schedules/cosine.rs:10-40 with
offset s, schedules/scaled.rs:9-40: betas linear in sqrt space), DDPM ancestral sampler
(samplers/ddpm.rs:11-80), DDIM with eta (samplers/ddim.rs:11-80), guidance (guidance.rs:7-40),
training loss (diffusion/losses.rs), sinusoidal time embeddings (unet/embeddings.rs).

Formulas are those of Ho et al. 2020 (DDPM), Nichol & Dhariwal 2021 (cosine schedule) and Song et al.
2021 (DDIM). Schedules are precomputed tensors on the model's device, so one sampling step is a few
fused elementwise ops plus the denoiser's forward.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..nn.layers import Linear
from ..nn.module import Module


class NoiseSchedule:
    """betas [T] and the derived alphas / cumulative products (float64 on the host, cast on use)."""

    def __init__(self, betas: torch.Tensor):
        self.betas = betas.to(torch.float64).clamp(1e-8, 0.999)
        self.alphas = 1.0 - self.betas
        self.alphas_cumprod = torch.cumprod(self.alphas, 0)
        self.timesteps = self.betas.numel()

    def at(self, name: str, t: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
        v = getattr(self, name).to(like.device)[t.to(like.device)].to(like.dtype)
        return v.view(-1, *([1] * (like.dim() - 1)))


class LinearSchedule(NoiseSchedule):
    def __init__(self, timesteps: int = 1000, beta_start: float = 1e-4, beta_end: float = 0.02):
        super().__init__(torch.linspace(beta_start, beta_end, timesteps, dtype=torch.float64))


class ScaledLinearSchedule(NoiseSchedule):
    def __init__(self, timesteps: int = 1000, beta_start: float = 0.00085, beta_end: float = 0.012):
        super().__init__(torch.linspace(beta_start ** 0.5, beta_end ** 0.5, timesteps, dtype=torch.float64) ** 2)


class CosineSchedule(NoiseSchedule):
    def __init__(self, timesteps: int = 1000, s: float = 0.008):
        x = torch.arange(timesteps + 1, dtype=torch.float64)
        f = torch.cos((x / timesteps + s) / (1 + s) * math.pi / 2) ** 2
        ac = f / f[0]
        super().__init__(1 - ac[1:] / ac[:-1])


def q_sample(schedule: NoiseSchedule, x0, t, noise):
    """x_t = sqrt(ᾱ_t) x0 + sqrt(1 − ᾱ_t) ε."""
    ac = schedule.at("alphas_cumprod", t, x0)
    return ac.sqrt() * x0 + (1 - ac).sqrt() * noise


def diffusion_loss(model, schedule: NoiseSchedule, x0, cond=None, generator=None):
    """Simple epsilon-prediction MSE at uniformly drawn timesteps."""
    t = torch.randint(0, schedule.timesteps, (x0.shape[0],), generator=generator, device="cpu").to(x0.device)
    noise = torch.randn(x0.shape, generator=generator, device="cpu", dtype=torch.float32).to(x0.device, x0.dtype)
    pred = model(q_sample(schedule, x0, t, noise), t, cond)
    return torch.nn.functional.mse_loss(pred.float(), noise.float())


def guided_eps(model, x, t, cond, guidance_scale: float):
    """Classifier-free guidance: ε_uncond + w (ε_cond − ε_uncond); ``cond=None`` is the null condition."""
    if cond is None or guidance_scale == 1.0:
        return model(x, t, cond)
    e_u, e_c = model(x, t, None), model(x, t, cond)
    return e_u + guidance_scale * (e_c - e_u)


class DdpmSampler:
    def __init__(self, schedule: NoiseSchedule):
        self.s = schedule

    @classmethod
    def from_schedule(cls, schedule):
        return cls(schedule)

    def step(self, eps, t: int, x, generator=None):
        s = self.s
        tt = torch.full((x.shape[0],), t, dtype=torch.long)
        a, ac, b = s.at("alphas", tt, x), s.at("alphas_cumprod", tt, x), s.at("betas", tt, x)
        mean = (x - b / (1 - ac).sqrt() * eps) / a.sqrt()
        if t == 0:
            return mean
        ac_prev = s.at("alphas_cumprod", tt - 1, x)
        var = b * (1 - ac_prev) / (1 - ac)
        z = torch.randn(x.shape, generator=generator, device="cpu", dtype=torch.float32).to(x.device, x.dtype)
        return mean + var.sqrt() * z

    @torch.no_grad()
    def sample(self, model, shape, device=None, cond=None, guidance_scale: float = 1.0, generator=None, dtype=None):
        x = torch.randn(shape, generator=generator, device="cpu").to(device=device, dtype=dtype or torch.float32)
        for t in range(self.s.timesteps - 1, -1, -1):
            tt = torch.full((shape[0],), t, dtype=torch.long, device=x.device)
            x = self.step(guided_eps(model, x, tt, cond, guidance_scale), t, x, generator)
        return x


class DdimSampler:
    """Deterministic for eta = 0; ``num_steps`` evenly spaced timesteps."""

    def __init__(self, schedule: NoiseSchedule, eta: float = 0.0):
        self.s, self.eta = schedule, eta

    @classmethod
    def from_schedule(cls, schedule, eta=0.0):
        return cls(schedule, eta)

    @torch.no_grad()
    def sample(self, model, shape, num_steps: int = 50, device=None, cond=None, guidance_scale: float = 1.0,
               generator=None, x=None, dtype=None):
        T = self.s.timesteps
        ts = torch.linspace(T - 1, 0, num_steps).round().long().tolist()
        if x is None:
            x = torch.randn(shape, generator=generator, device="cpu").to(device=device, dtype=dtype or torch.float32)
        ac_all = self.s.alphas_cumprod
        for i, t in enumerate(ts):
            tt = torch.full((shape[0],), t, dtype=torch.long, device=x.device)
            eps = guided_eps(model, x, tt, cond, guidance_scale)
            ac = float(ac_all[t])
            ac_prev = float(ac_all[ts[i + 1]]) if i + 1 < len(ts) else 1.0
            x0 = (x - math.sqrt(1 - ac) * eps) / math.sqrt(ac)
            sigma = self.eta * math.sqrt((1 - ac_prev) / (1 - ac) * (1 - ac / ac_prev))
            x = math.sqrt(ac_prev) * x0 + math.sqrt(max(0.0, 1 - ac_prev - sigma ** 2)) * eps
            if sigma > 0:
                x = x + sigma * torch.randn(x.shape, generator=generator, device="cpu").to(x.device, x.dtype)
        return x


def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
    a = t.float()[:, None] * freqs[None]
    return torch.cat([torch.cos(a), torch.sin(a)], -1)


class MlpDenoiser(Module):
    """ε_θ(x_t, t, c) for flat data: [x, time embedding, class embedding] -> SiLU MLP -> ε.
    Class index ``num_classes`` is the null condition used by guidance training."""

    def __init__(self, data_dim: int, hidden: int = 128, time_dim: int = 32, num_classes: int = 0, device=None,
                 dtype=None):
        super().__init__()
        self.time_dim, self.num_classes = time_dim, num_classes
        self.cls = torch.nn.Embedding(num_classes + 1, time_dim, device=device, dtype=dtype) if num_classes else None
        self.l1 = Linear(data_dim + time_dim, hidden, True, device, dtype)
        self.l2 = Linear(hidden, hidden, True, device, dtype)
        self.l3 = Linear(hidden, data_dim, True, device, dtype)

    def forward(self, x, t, cond=None):
        e = timestep_embedding(t, self.time_dim).to(x.dtype)
        if self.cls is not None:
            c = cond if cond is not None else torch.full((x.shape[0],), self.num_classes, device=x.device)
            e = e + self.cls(c)
        h = torch.nn.functional.silu(self.l1(torch.cat([x, e], -1)))
        return self.l3(torch.nn.functional.silu(self.l2(h)))


class EulerAncestralSampler:
    """Ancestral sampling in the sigma parameterisation (sigma_t = sqrt((1 − ᾱ_t) / ᾱ_t)), Euler steps
    with noise re-injected at each step (Karras et al. 2022, "ancestral" variant; reference
    samplers/ancestral.rs). ``eta = 0`` gives the deterministic Euler sampler."""

    def __init__(self, schedule: NoiseSchedule, eta: float = 1.0):
        self.s, self.eta = schedule, eta

    @torch.no_grad()
    def sample(self, model, shape, num_steps: int = 50, device=None, cond=None, guidance_scale: float = 1.0,
               generator=None, dtype=None):
        ac = self.s.alphas_cumprod
        ts = torch.linspace(self.s.timesteps - 1, 0, num_steps).round().long().tolist()
        sig = [math.sqrt((1 - float(ac[t])) / float(ac[t])) for t in ts] + [0.0]
        x = torch.randn(shape, generator=generator, device="cpu").to(device=device, dtype=dtype or torch.float32)
        x = x * math.sqrt(sig[0] ** 2 + 1)
        for i, t in enumerate(ts):
            s0, s1 = sig[i], sig[i + 1]
            tt = torch.full((shape[0],), t, dtype=torch.long, device=x.device)
            eps = guided_eps(model, x / math.sqrt(s0 ** 2 + 1), tt, cond, guidance_scale)
            s_up = min(s1, self.eta * math.sqrt(max(0.0, s1 ** 2 * (s0 ** 2 - s1 ** 2) / max(s0 ** 2, 1e-12))))
            s_down = math.sqrt(max(0.0, s1 ** 2 - s_up ** 2))
            x = x + eps * (s_down - s0)
            if s_up > 0:
                x = x + s_up * torch.randn(x.shape, generator=generator, device="cpu").to(x.device, x.dtype)
        return x


# ------------------------------------------------------------------ the reference's entry points
# crates/brain-diffusion/src: unet/embeddings.rs (sinusoidal_timestep_embedding), diffusion/losses.rs
# (eps_loss), diffusion/train.rs (training_step), utils.rs (linspace_timesteps, extract_at_t),
# diffusion/mod.rs + impl.rs (DiffusionModel / DiffusionRunner: denoiser + schedule + sampler),
# guidance.rs (GuidanceConfig).
sinusoidal_timestep_embedding = timestep_embedding


def eps_loss(pred_eps: torch.Tensor, true_eps: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.mse_loss(pred_eps.float(), true_eps.float())


def linspace_timesteps(num_train_steps: int, num_steps: int) -> torch.Tensor:
    """Descending sampling timesteps spread evenly over [0, num_train_steps - 1]."""
    return torch.linspace(num_train_steps - 1, 0, num_steps).round().long()


def extract_at_t(values: torch.Tensor, t: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """values[t] reshaped to broadcast against ``like`` ([B, 1, 1, ...])."""
    v = values.to(like.device)[t.to(like.device)].to(like.dtype)
    return v.view(-1, *([1] * (like.dim() - 1)))


def training_step(model, schedule: NoiseSchedule, optimizer, x0, cond=None, generator=None,
                  cond_drop_prob: float = 0.0) -> float:
    """One epsilon-prediction update; with ``cond_drop_prob`` the condition is dropped for the whole
    batch with that probability (training for classifier-free guidance)."""
    if cond is not None and cond_drop_prob > 0:
        u = float(torch.rand((), generator=generator))
        cond = None if u < cond_drop_prob else cond
    loss = diffusion_loss(model, schedule, x0, cond, generator)
    optimizer.zero_grad()
    loss.backward()
    optimizer.step()
    return float(loss.detach())


@dataclass
class GuidanceConfig:
    scale: float = 1.0
    cond_drop_prob: float = 0.1


class DiffusionModel:
    """A denoiser with its noise schedule and a sampler: ``train_step(x0)`` and ``sample(shape)``."""

    def __init__(self, denoiser, schedule: NoiseSchedule | None = None, sampler: str = "ddim",
                 guidance: GuidanceConfig | None = None):
        self.denoiser = denoiser
        self.schedule = schedule or LinearSchedule()
        self.sampler = {"ddpm": DdpmSampler, "ddim": DdimSampler, "euler_a": EulerAncestralSampler}[sampler](self.schedule)
        self.guidance = guidance or GuidanceConfig()

    def train_step(self, optimizer, x0, cond=None, generator=None) -> float:
        return training_step(self.denoiser, self.schedule, optimizer, x0, cond, generator,
                             self.guidance.cond_drop_prob if cond is not None else 0.0)

    @torch.no_grad()
    def sample(self, shape, device=None, cond=None, generator=None, **kw):
        return self.sampler.sample(self.denoiser, shape, device=device, cond=cond,
                                   guidance_scale=self.guidance.scale, generator=generator, **kw)


DiffusionRunner = DiffusionModel
