"""Loss-landscape probes: filter-normalised random directions and 1-D / 2-D loss surfaces around the
current weights (Li et al. 2018).

Reference: crates/brain-optim/src/loss_landscape.rs (LossLandscapeConfig, create_filter_normalized_direction,
interpolate_1d). The reference's direction is a constant vector rescaled to the parameter's norm; here it
is Gaussian and normalised per filter (each output row gets the norm of the matching weight row), the
construction the method prescribes, with the constant direction available as ``kind="constant"``.
Surfaces are evaluated by moving the model's weights in place and restoring them afterwards.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class LossLandscapeConfig:
    num_points: int = 21
    x_min: float = -1.0
    x_max: float = 1.0
    y_min: float = -1.0
    y_max: float = 1.0
    filter_normalized: bool = True


def create_filter_normalized_direction(param: torch.Tensor, kind: str = "gaussian", generator=None) -> torch.Tensor:
    """A direction shaped like ``param``: per filter (row of a >= 2-D weight) its norm equals that row's
    norm; 1-D parameters (biases, norms) get a zero direction, as the method does."""
    if kind == "constant":
        d = torch.ones_like(param, dtype=torch.float64)
        return (d * param.double().norm() / d.norm().clamp_min(1e-12)).to(param.dtype)
    if param.dim() < 2:
        return torch.zeros_like(param)
    d = torch.randn(param.shape, generator=generator, dtype=torch.float64).to(param.device)
    p2, d2 = param.double().reshape(param.shape[0], -1), d.reshape(param.shape[0], -1)
    d2 = d2 * (p2.norm(dim=1, keepdim=True) / d2.norm(dim=1, keepdim=True).clamp_min(1e-12))
    return d2.reshape(param.shape).to(param.dtype)


def interpolate_1d(theta0, direction, alpha: float):
    """theta0 + alpha direction, tensor by tensor."""
    return [p + alpha * d for p, d in zip(theta0, direction)]


@torch.no_grad()
def loss_surface(model, loss_fn, config: LossLandscapeConfig | None = None, two_d: bool = False, generator=None):
    """Loss along one (or two) filter-normalised directions: returns (alphas, losses [n]) or
    (alphas, betas, losses [n, n]); ``loss_fn(model)`` evaluates the current weights."""
    c = config or LossLandscapeConfig()
    params = [p for p in model.parameters()]
    theta0 = [p.detach().clone() for p in params]
    mk = (lambda p: create_filter_normalized_direction(p, generator=generator)) if c.filter_normalized else \
        (lambda p: torch.randn(p.shape, generator=generator).to(p))
    d1 = [mk(p) for p in params]
    d2 = [mk(p) for p in params] if two_d else None
    xs = torch.linspace(c.x_min, c.x_max, c.num_points)
    ys = torch.linspace(c.y_min, c.y_max, c.num_points)
    try:
        if not two_d:
            out = torch.empty(c.num_points)
            for i, a in enumerate(xs.tolist()):
                for p, t0, d in zip(params, theta0, d1):
                    p.copy_(t0 + a * d)
                out[i] = float(loss_fn(model))
            return xs, out
        out = torch.empty(c.num_points, c.num_points)
        for i, a in enumerate(xs.tolist()):
            for j, b in enumerate(ys.tolist()):
                for p, t0, da, db in zip(params, theta0, d1, d2):
                    p.copy_(t0 + a * da + b * db)
                out[i, j] = float(loss_fn(model))
        return xs, ys, out
    finally:
        for p, t0 in zip(params, theta0):
            p.copy_(t0)
