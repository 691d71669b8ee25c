"""Weight initialisers (crates/brain-nn/src/init/*.rs): kaiming/xavier uniform+normal, normal,
uniform, zeros/ones, orthogonal, scaled residual init and the seeded N(0, std) used by the
benchmark configurations. All take an optional ``torch.Generator`` for reproducibility."""
from __future__ import annotations

import math

import torch


def _fan(t: torch.Tensor):
    if t.dim() < 2:
        return t.numel(), t.numel()
    recept = t[0][0].numel() if t.dim() > 2 else 1
    return t.shape[1] * recept, t.shape[0] * recept


@torch.no_grad()
def _fill(t, sample):
    tmp = sample.to(dtype=torch.float32)
    t.copy_(tmp.to(device=t.device, dtype=t.dtype))
    return t


def normal_(t, mean=0.0, std=0.02, generator=None):
    return _fill(t, torch.randn(t.shape, generator=generator) * std + mean)


def uniform_(t, a=-1.0, b=1.0, generator=None):
    return _fill(t, torch.rand(t.shape, generator=generator) * (b - a) + a)


def zeros_(t):
    with torch.no_grad():
        return t.zero_()


def ones_(t):
    with torch.no_grad():
        return t.fill_(1.0)


def kaiming_uniform_(t, a=math.sqrt(5), generator=None):
    fan_in, _ = _fan(t)
    gain = math.sqrt(2.0 / (1 + a * a))
    bound = gain * math.sqrt(3.0 / max(1, fan_in))
    return uniform_(t, -bound, bound, generator)


def kaiming_normal_(t, generator=None):
    fan_in, _ = _fan(t)
    return normal_(t, 0.0, math.sqrt(2.0 / max(1, fan_in)), generator)


def xavier_uniform_(t, gain=1.0, generator=None):
    fan_in, fan_out = _fan(t)
    bound = gain * math.sqrt(6.0 / max(1, fan_in + fan_out))
    return uniform_(t, -bound, bound, generator)


def xavier_normal_(t, gain=1.0, generator=None):
    fan_in, fan_out = _fan(t)
    return normal_(t, 0.0, gain * math.sqrt(2.0 / max(1, fan_in + fan_out)), generator)


def orthogonal_(t, gain=1.0, generator=None):
    rows, cols = t.shape[0], t.numel() // t.shape[0]
    a = torch.randn(max(rows, cols), min(rows, cols), generator=generator)
    q, r = torch.linalg.qr(a)
    q = q * torch.sign(torch.diagonal(r))
    if rows < cols:
        q = q.t()
    return _fill(t, (gain * q[:rows, :cols]).reshape(t.shape))


def scaled_residual_(t, num_layers, std=0.02, generator=None):
    """N(0, std / sqrt(2 * num_layers)) for residual output projections (GPT-2 style)."""
    return normal_(t, 0.0, std / math.sqrt(2.0 * num_layers), generator)


@torch.no_grad()
def init_normal_(module: torch.nn.Module, std: float = 0.02, seed: int = 0) -> None:
    """Seeded N(0, std) for every weight matrix / embedding; norms to one, biases to zero.

    Samples are drawn on the parameter's own device from a generator seeded with ``seed`` (one
    stream over the parameters in registration order), so an 8B-parameter model initialises in
    seconds on a GPU and identically on every rank.
    """
    gens = {}
    for name, p in module.named_parameters():
        if p.dim() >= 2:
            dev = p.device
            g = gens.get(str(dev))
            if g is None:
                g = torch.Generator(device=dev).manual_seed(seed)
                gens[str(dev)] = g
            p.copy_((torch.randn(p.shape, generator=g, device=dev, dtype=torch.float32) * std).to(p.dtype))
        elif name.endswith("bias"):
            zeros_(p)
        else:
            ones_(p)


def calculate_fan(shape) -> tuple[int, int]:
    """(fan_in, fan_out) of a weight shape: [out, in, *kernel] -> (in * k, out * k); 1-D -> (n, n)."""
    shape = tuple(shape)
    if len(shape) < 2:
        n = shape[0] if shape else 1
        return n, n
    rf = 1
    for d in shape[2:]:
        rf *= d
    return shape[1] * rf, shape[0] * rf


def scaled_residual_init(weight: torch.Tensor, num_residual_layers: int) -> torch.Tensor:
    """weight / sqrt(2 L): the GPT-2 scaling of residual-branch output projections."""
    return weight * (1.0 / math.sqrt(2.0 * max(num_residual_layers, 1)))


def zero_init_last_layer(shape, dtype=torch.float32, device=None) -> torch.Tensor:
    """A zero weight, so a residual block starts as the identity."""
    return torch.zeros(tuple(shape), dtype=dtype, device=device)
