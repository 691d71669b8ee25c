"""Core layers with the reference's names, running on the sm_100a ops.

Linear ([out, in] weight, kaiming-uniform init, optional zero bias; crates/brain-nn/src/layers/linear.rs:13-63),
Embedding (crates/brain-nn/src/layers/embedding.rs:34-60), LayerNorm / RMSNorm
(crates/brain-nn/src/normalization/*.rs — here differentiable end to end, where the reference's
LayerNorm module breaks the tape), MultiheadAttention with q/k/v/out projections
(crates/brain-nn/src/layers/multihead.rs:40-149), GroupedQueryAttention, FeedForward (SwiGLU /
GELU), Dropout and the usual activation modules.
"""
from __future__ import annotations

import math

import torch

from .. import ops
from . import init as _init
from .module import Module


class Linear(Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None,
                 generator=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = torch.nn.Parameter(torch.empty(out_features, in_features, device=device, dtype=dtype))
        self.bias = torch.nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype)) if bias else None
        _init.kaiming_uniform_(self.weight, generator=generator)

    def forward(self, x, residual=None):
        return ops.linear(x, self.weight, self.bias, residual)

    def extra_repr(self):
        return f"in={self.in_features}, out={self.out_features}, bias={self.bias is not None}"


class Embedding(Module):
    def __init__(self, num_embeddings: int, embedding_dim: int, device=None, dtype=None, generator=None):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.empty(num_embeddings, embedding_dim, device=device, dtype=dtype))
        _init.normal_(self.weight, 0.0, 1.0, generator)

    def forward(self, ids):
        return ops.embedding(ids, self.weight)

    forward_indices = forward


class RMSNorm(Module):
    def __init__(self, dim: int, eps: float = 1e-6, device=None, dtype=None):
        super().__init__()
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.ones(dim, device=device, dtype=dtype))

    def forward(self, x):
        return ops.rms_norm(x, self.weight, self.eps)


class LayerNorm(Module):
    def __init__(self, dim: int, eps: float = 1e-5, bias: bool = True, device=None, dtype=None):
        super().__init__()
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.ones(dim, device=device, dtype=dtype))
        self.bias = torch.nn.Parameter(torch.zeros(dim, device=device, dtype=dtype)) if bias else None

    def forward(self, x):
        return ops.layer_norm(x, self.weight, self.bias, self.eps)


class Dropout(Module):
    def __init__(self, p: float = 0.1):
        super().__init__()
        self.p = p

    def forward(self, x):
        return torch.nn.functional.dropout(x, self.p, self.training)


class GELU(Module):
    """tanh-approximate GELU (the reference's only GELU, crates/brain-core/src/tensor/math.rs:284-287)."""

    def forward(self, x):
        return ops.gelu(x)


class SiLU(Module):
    def forward(self, x):
        return torch.nn.functional.silu(x)


Swish = SiLU


class ReLU(Module):
    def forward(self, x):
        return torch.relu(x)


class LeakyReLU(Module):
    def __init__(self, negative_slope=0.01):
        super().__init__()
        self.negative_slope = negative_slope

    def forward(self, x):
        return torch.nn.functional.leaky_relu(x, self.negative_slope)


class Tanh(Module):
    def forward(self, x):
        return torch.tanh(x)


class Sigmoid(Module):
    def forward(self, x):
        return torch.sigmoid(x)


class Softmax(Module):
    def __init__(self, dim=-1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return torch.softmax(x.float() - x.float().amax(self.dim, keepdim=True), self.dim).to(x.dtype)


class LogSoftmax(Softmax):
    def forward(self, x):
        return torch.log_softmax(x.float(), self.dim).to(x.dtype)


class SwiGLU(Module):
    """silu(gate) * up over a fused [..., 2F] input."""

    def forward(self, gu):
        return ops.swiglu(gu)


class ELU(Module):
    def __init__(self, alpha=1.0):
        super().__init__()
        self.alpha = alpha

    def forward(self, x):
        return torch.nn.functional.elu(x, self.alpha)


class SELU(Module):
    def forward(self, x):
        return torch.nn.functional.selu(x)


class Mish(Module):
    def forward(self, x):
        return torch.nn.functional.mish(x)


class Softplus(Module):
    def forward(self, x):
        return torch.nn.functional.softplus(x)


class Hardswish(Module):
    def forward(self, x):
        return torch.nn.functional.hardswish(x)


class Hardsigmoid(Module):
    def forward(self, x):
        return torch.nn.functional.hardsigmoid(x)


class PReLU(Module):
    def __init__(self, num_parameters=1, init=0.25):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.full((num_parameters,), init))

    def forward(self, x):
        return torch.nn.functional.prelu(x, self.weight.to(x.dtype))


class GLU(Module):
    def __init__(self, dim=-1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return torch.nn.functional.glu(x, self.dim)


class QuickGELU(Module):
    def forward(self, x):
        return x * torch.sigmoid(1.702 * x)


class FeedForward(Module):
    """Transformer FFN: gated (SwiGLU over a fused gate/up weight) or plain (GELU)."""

    def __init__(self, dim: int, hidden: int, gated: bool = True, bias: bool = False, device=None, dtype=None,
                 act: str = "gelu", fused_gelu: bool = False):
        super().__init__()
        self.gated = gated
        self.act = act
        # GELU inside the GEMM epilogues (``ops.gelu_mlp``). Off by default: at d_model 768 the four epilogue
        # warps of the GEMM become the bottleneck and the fused pair measured slower than GEMM + activation.
        self.fused_gelu = fused_gelu
        if gated:
            self.gate_up = Linear(dim, 2 * hidden, bias=bias, device=device, dtype=dtype)
        else:
            self.up = Linear(dim, hidden, bias=bias, device=device, dtype=dtype)
        self.down = Linear(hidden, dim, bias=bias, device=device, dtype=dtype)

    def forward(self, x, residual=None):
        if self.gated:
            if self.down.bias is None:
                return ops.swiglu_linear(self.gate_up(x), self.down.weight, residual)
            return self.down(ops.swiglu(self.gate_up(x)), residual)
        if self.act == "gelu" and self.fused_gelu:
            return ops.gelu_mlp(x, self.up.weight, self.up.bias, self.down.weight, self.down.bias, residual)
        h = self.up(x)
        h = torch.relu(h) if self.act == "relu" else ops.gelu(h)
        return self.down(h, residual)


class MultiheadAttention(Module):
    """Multi-head (or grouped-query, when num_kv_heads < num_heads) self-attention.

    One fused [q; k; v] projection feeds the flash-attention kernel directly through strides.
    ``causal`` selects the decoder mask; RoPE is applied when a rope table is passed.
    """

    def __init__(self, dim: int, num_heads: int, num_kv_heads: int | None = None, bias: bool = True,
                 causal: bool = False, device=None, dtype=None):
        super().__init__()
        self.dim, self.num_heads = dim, num_heads
        self.num_kv_heads = num_kv_heads or num_heads
        self.head_dim = dim // num_heads
        self.causal = causal
        qkv_out = (self.num_heads + 2 * self.num_kv_heads) * self.head_dim
        self.qkv = Linear(dim, qkv_out, bias=bias, device=device, dtype=dtype)
        self.out = Linear(num_heads * self.head_dim, dim, bias=bias, device=device, dtype=dtype)

    def forward(self, x, rope_table=None, residual=None, causal=None):
        c = self.causal if causal is None else causal
        qkv = self.qkv(x)
        o = ops.qkv_attention(qkv, self.num_heads, self.num_kv_heads, rope_table, causal=c)
        return self.out(o, residual)


class GroupedQueryAttention(MultiheadAttention):
    def __init__(self, dim, num_heads, num_kv_heads, bias=False, causal=True, device=None, dtype=None):
        super().__init__(dim, num_heads, num_kv_heads, bias, causal, device, dtype)


class MultiQueryAttention(MultiheadAttention):
    def __init__(self, dim, num_heads, bias=False, causal=True, device=None, dtype=None):
        super().__init__(dim, num_heads, 1, bias, causal, device, dtype)


def scaled_dot_product_attention(q, k, v, causal=False, scale=None):
    """[B, S, H, D] attention (reference: crates/brain-transformer/src/attention/scaled.rs:41-139)."""
    return ops.flash_attention(q, k, v, causal, scale)


class Conv2d(torch.nn.Conv2d, Module):
    """2-D convolution (cuDNN through PyTorch; crates/brain-nn/src/layers/conv*.rs)."""


class Conv1d(torch.nn.Conv1d, Module):
    pass


class ConvTranspose2d(torch.nn.ConvTranspose2d, Module):
    pass


class MaxPool2d(torch.nn.MaxPool2d, Module):
    pass


class AvgPool2d(torch.nn.AvgPool2d, Module):
    pass


class AdaptiveAvgPool2d(torch.nn.AdaptiveAvgPool2d, Module):
    pass


class BatchNorm2d(torch.nn.BatchNorm2d, Module):
    pass


class GroupNorm(torch.nn.GroupNorm, Module):
    pass


class InstanceNorm2d(torch.nn.InstanceNorm2d, Module):
    pass


class BatchNorm1d(torch.nn.BatchNorm1d, Module):
    pass


class InstanceNorm1d(torch.nn.InstanceNorm1d, Module):
    pass


class Flatten(torch.nn.Flatten, Module):
    pass


class PixelShuffle(torch.nn.PixelShuffle, Module):
    pass


class LSTM(torch.nn.LSTM, Module):
    pass


class GRU(torch.nn.GRU, Module):
    pass


class RNN(torch.nn.RNN, Module):
    pass


class Bilinear(torch.nn.Bilinear, Module):
    pass


def num_params(m: torch.nn.Module) -> int:
    return sum(p.numel() for p in m.parameters())




# ------------------------------------------------------------------ further activations (crates/brain-nn/src/activations/extra.rs, extended.rs)
class CELU(Module):
    """x for x > 0, alpha (exp(x / alpha) - 1) otherwise (alpha > 0)."""

    def __init__(self, alpha: float = 1.0):
        super().__init__()
        if alpha <= 0:
            raise ValueError("CELU alpha must be positive")
        self.alpha = alpha

    def forward(self, x):
        return torch.where(x > 0, x, self.alpha * torch.expm1(x / self.alpha))


class HardShrink(Module):
    """x where |x| > lambda, else 0."""

    def __init__(self, lambd: float = 0.5):
        super().__init__()
        self.lambd = lambd

    def forward(self, x):
        return torch.where(x.abs() > self.lambd, x, torch.zeros_like(x))


class SoftShrink(Module):
    """x - lambda above lambda, x + lambda below -lambda, else 0."""

    def __init__(self, lambd: float = 0.5):
        super().__init__()
        self.lambd = lambd

    def forward(self, x):
        return torch.sign(x) * (x.abs() - self.lambd).clamp_min(0)


class Shrink(Module):
    """ONNX Shrink: x - bias above lambda, x + bias below -lambda, else 0."""

    def __init__(self, lambd: float = 0.5, bias: float = 0.5):
        super().__init__()
        self.lambd, self.bias = lambd, bias

    def forward(self, x):
        return torch.where(x > self.lambd, x - self.bias, torch.where(x < -self.lambd, x + self.bias,
                                                                      torch.zeros_like(x)))


class TanhShrink(Module):
    def forward(self, x):
        return x - torch.tanh(x)


class ThresholdedReLU(Module):
    """x where x > theta, else 0."""

    def __init__(self, theta: float = 1.0):
        super().__init__()
        self.theta = theta

    def forward(self, x):
        return torch.where(x > self.theta, x, torch.zeros_like(x))


class Softmin(Module):
    def __init__(self, dim: int = -1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return torch.softmax(-x, self.dim)


def quiet_softmax(x: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Softmax of x / (1 + exp(x)) along ``dim`` (the reference's "quiet" variant damps large logits)."""
    return torch.softmax(x / (1.0 + torch.exp(x)), dim)


class QuietSoftmax(Module):
    def __init__(self, dim: int = -1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return quiet_softmax(x, self.dim)


class FusedDropout(Module):
    """dropout(x) + residual in one call (inverted dropout; identity in eval)."""

    def __init__(self, p: float = 0.1):
        super().__init__()
        self.p = p

    def forward_add(self, x, residual):
        return torch.nn.functional.dropout(x, self.p, self.training) + residual

    forward = forward_add


class SequentialNamed(Module):
    """Sequential container with explicit child names (``[(name, module), ...]``)."""

    def __init__(self, named):
        super().__init__()
        self._order = []
        for name, m in named:
            self.add_module(name, m)
            self._order.append(name)

    def forward(self, x):
        for name in self._order:
            x = getattr(self, name)(x)
        return x


# The reference's spellings (crates/brain-transformer/src/attention/multi_head.rs, ffn/mod.rs).
MultiHeadAttention = MultiheadAttention
FeedForwardNetwork = FeedForward


__all__ = [n for n in dir() if not n.startswith("_") and n[0].isupper()] + ["scaled_dot_product_attention",
                                                                             "num_params", "math", "quiet_softmax"]
