"""Closed-form vector-Jacobian products with the reference's names (``grad_relu(x, g)``,
``grad_matmul_a(a, b, g)``, ``grad_layernorm(x, gamma, g, eps)`` ...), for callers that build their own
backward passes or check one. Each is the analytic derivative written with tensor ops, so it runs
on whatever device its inputs are on; the tests compare every one against torch autograd.

Reference: crates/brain-autograd/src/grad_fns/arith.rs (add/sub/mul/div/pow/matmul), nnops.rs
(exp/log/sqrt/relu/sigmoid/tanh/softmax/log_softmax), composite.rs (layer norm over the whole input,
scaled dot-product attention), loss_grad.rs (MSE 2 g / N, cross-entropy and BCE with logits g / N),
ops/activation_grad.rs (tanh-GELU, leaky ReLU, SiLU), ops/broadcast_grad.rs (unbroadcast),
ops/reduction_grad.rs, ops/tensor_grad.rs, ops/index_grad.rs (embedding), ops/linalg_grad.rs (inv, det),
ops/pool_grad.rs, ops/conv_grad.rs, ops/quant_grad.rs (straight-through within [min, max]),
ops/sparse_grad.rs, ops/fft_grad.rs.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def unbroadcast(g: torch.Tensor, target_shape) -> torch.Tensor:
    """Sum g over the dimensions that broadcasting added or expanded from size 1."""
    target_shape = tuple(target_shape)
    while g.dim() > len(target_shape):
        g = g.sum(0)
    for i, s in enumerate(target_shape):
        if s == 1 and g.shape[i] != 1:
            g = g.sum(i, keepdim=True)
    return g


grad_of_broadcast_to = unbroadcast


def grad_add_a(a, b, g):
    return unbroadcast(g, a.shape)


def grad_add_b(a, b, g):
    return unbroadcast(g, b.shape)


def grad_sub_a(a, b, g):
    return unbroadcast(g, a.shape)


def grad_sub_b(a, b, g):
    return unbroadcast(-g, b.shape)


def grad_mul_a(a, b, g):
    return unbroadcast(g * b, a.shape)


def grad_mul_b(a, b, g):
    return unbroadcast(g * a, b.shape)


def grad_div_a(a, b, g):
    return unbroadcast(g / b, a.shape)


def grad_div_b(a, b, g):
    return unbroadcast(-g * a / (b * b), b.shape)


def grad_pow_a(a, b, g):
    return unbroadcast(g * b * a.pow(b - 1), a.shape)


def grad_pow_b(a, b, g):
    return unbroadcast(g * a.pow(b) * torch.log(a), b.shape)


def grad_matmul_a(a, b, g):
    return g @ b.transpose(-1, -2)


def grad_matmul_b(a, b, g):
    return a.transpose(-1, -2) @ g


def grad_exp(x, g):
    return g * torch.exp(x)


def grad_log(x, g):
    return g / x


def grad_sqrt(x, g):
    return g * 0.5 / torch.sqrt(x)


def grad_relu(x, g):
    return g * (x > 0).to(g.dtype)


def grad_sigmoid(x, g):
    s = torch.sigmoid(x)
    return g * s * (1 - s)


def grad_tanh(x, g):
    t = torch.tanh(x)
    return g * (1 - t * t)


def grad_softmax(x, g, axis: int = -1):
    s = torch.softmax(x, axis)
    return s * (g - (g * s).sum(axis, keepdim=True))


def grad_log_softmax(x, g, axis: int = -1):
    return g - torch.softmax(x, axis) * g.sum(axis, keepdim=True)


def grad_gelu(x, g):
    """Derivative of the tanh approximation 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    c = math.sqrt(2.0 / math.pi)
    t = torch.tanh(c * (x + 0.044715 * x ** 3))
    return g * (0.5 * (1 + t) + 0.5 * x * (1 - t * t) * c * (1 + 3 * 0.044715 * x * x))


def grad_leaky_relu(x, g, negative_slope: float = 0.01):
    return g * torch.where(x > 0, torch.ones_like(x), torch.full_like(x, negative_slope))


def grad_silu(x, g):
    s = torch.sigmoid(x)
    return g * s * (1 + x * (1 - s))


def grad_layernorm(x, gamma, g, eps: float = 1e-5, normalized_dims: int | None = None):
    """(dx, dgamma, dbeta) of y = gamma * (x - mean) / sqrt(var + eps) + beta, normalising over the last
    ``normalized_dims`` dimensions (all of them by default, as the reference's composite does)."""
    nd = x.dim() if normalized_dims is None else normalized_dims
    dims = tuple(range(x.dim() - nd, x.dim()))
    mean = x.mean(dims, keepdim=True)
    xc = x - mean
    rstd = torch.rsqrt((xc * xc).mean(dims, keepdim=True) + eps)
    xhat = xc * rstd
    gx = g * gamma
    dx = rstd * (gx - gx.mean(dims, keepdim=True) - xhat * (gx * xhat).mean(dims, keepdim=True))
    batch_dims = tuple(range(x.dim() - nd))
    dgamma = (g * xhat).sum(batch_dims) if batch_dims else g * xhat
    dbeta = g.sum(batch_dims) if batch_dims else g.clone()
    return dx, dgamma, dbeta


def grad_scaled_dot_product_attention(q, k, v, g):
    """(dq, dk, dv) of softmax(q k^T / sqrt(d)) v for [..., S, d] operands (no mask)."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    p = torch.softmax((q @ k.transpose(-1, -2)) * scale, -1)
    dv = p.transpose(-1, -2) @ g
    dp = g @ v.transpose(-1, -2)
    ds = p * (dp - (dp * p).sum(-1, keepdim=True))
    return (ds @ k) * scale, (ds.transpose(-1, -2) @ q) * scale, dv


def grad_mse_loss(pred, target, g: float = 1.0):
    return (pred - target) * (2.0 * g / pred.numel())


def grad_cross_entropy_logits(logits, target_indices, g: float = 1.0):
    """(softmax(logits) - onehot) g / batch, over the last dimension; indices past the classes add no
    one-hot term."""
    C = logits.shape[-1]
    sm = torch.softmax(logits.reshape(-1, C), -1)
    t = torch.as_tensor(target_indices, device=logits.device).reshape(-1).long()
    ok = t < C
    sm[torch.arange(sm.shape[0], device=logits.device)[ok], t[ok]] -= 1.0
    return (sm * (g / sm.shape[0])).reshape(logits.shape)


def grad_bce_with_logits(logits, targets, g: float = 1.0):
    return (torch.sigmoid(logits) - targets) * (g / logits.numel())


def grad_sum_axis(g, orig_shape, axis: int):
    return g.unsqueeze(axis).expand(tuple(orig_shape)) if g.dim() < len(orig_shape) else g.expand(tuple(orig_shape))


def grad_mean_axis(g, orig_shape, axis: int):
    return grad_sum_axis(g, orig_shape, axis) / orig_shape[axis]


def grad_reshape(g, orig_shape):
    return g.reshape(tuple(orig_shape))


def grad_transpose(g, dim0: int, dim1: int):
    return g.transpose(dim0, dim1)


def grad_permute(g, dims):
    inv = [0] * len(dims)
    for i, d in enumerate(dims):
        inv[d] = i
    return g.permute(*inv)


def grad_embedding(g, num_embeddings: int, embedding_dim: int, indices):
    """Scatter-add of the output rows into a [num_embeddings, embedding_dim] weight gradient."""
    idx = torch.as_tensor(indices, device=g.device).reshape(-1).long()
    out = torch.zeros(num_embeddings, embedding_dim, device=g.device, dtype=g.dtype)
    return out.index_add_(0, idx, g.reshape(-1, embedding_dim))


def grad_inv(a_inv, grad_output):
    """d(A^-1): -A^-T G A^-T."""
    t = a_inv.transpose(-1, -2)
    return -(t @ grad_output @ t)


def grad_det(a, det_val, g: float = 1.0):
    """d det(A) = g det(A) A^-T."""
    return g * det_val * torch.linalg.inv(a).transpose(-1, -2)


def grad_conv2d(inp, weight, grad_output, stride=(1, 1), padding=(0, 0), dilation=(1, 1)):
    """(dinput, dweight, dbias) of a 2-D convolution (NCHW, OIHW)."""
    gi = torch.nn.grad.conv2d_input(inp.shape, weight, grad_output, stride, padding, dilation)
    gw = torch.nn.grad.conv2d_weight(inp, weight.shape, grad_output, stride, padding, dilation)
    return gi, gw, grad_output.sum((0, 2, 3))


def grad_conv_transpose2d(inp, weight, grad_output, stride=(1, 1), padding=(0, 0)):
    """(dinput, dweight) of conv_transpose2d: its input gradient is a forward convolution."""
    gi = F.conv2d(grad_output, weight, stride=stride, padding=padding)
    gw = torch.nn.grad.conv2d_weight(grad_output, weight.shape, inp, stride, padding)
    return gi, gw


def _vjp(fn, x, g):
    x = x.detach().requires_grad_(True)
    with torch.enable_grad():
        y = fn(x)
        (gx,) = torch.autograd.grad(y, x, g)
    return gx


def grad_avg_pool2d_ext(input_shape, grad_output, kernel_size, stride, padding=(0, 0)):
    x = torch.zeros(tuple(input_shape), device=grad_output.device, dtype=grad_output.dtype)
    return _vjp(lambda t: F.avg_pool2d(t, kernel_size, stride, padding), x, grad_output)


def grad_avg_pool2d(input_shape, grad_output, kernel_size):
    return grad_avg_pool2d_ext(input_shape, grad_output, kernel_size, kernel_size)


def grad_max_pool2d(inp, grad_output, kernel_size, stride, padding=(0, 0)):
    return _vjp(lambda t: F.max_pool2d(t, kernel_size, stride, padding), inp, grad_output)


def grad_adaptive_avg_pool2d(input_shape, grad_output, out_h: int, out_w: int):
    x = torch.zeros(tuple(input_shape), device=grad_output.device, dtype=grad_output.dtype)
    return _vjp(lambda t: F.adaptive_avg_pool2d(t, (out_h, out_w)), x, grad_output)


def grad_adaptive_max_pool2d(inp, grad_output, out_h: int, out_w: int):
    return _vjp(lambda t: F.adaptive_max_pool2d(t, (out_h, out_w)), inp, grad_output)


def grad_quantize_ste(x, g, min_val: float, max_val: float):
    """Straight-through: the gradient passes where min <= x <= max, zero outside."""
    return g * ((x >= min_val) & (x <= max_val)).to(g.dtype)


def grad_spmm_dense(sparse, dense_b, grad_output):
    """(d sparse values as a dense [R, C] matrix, d dense_b) of sparse @ dense_b."""
    a = sparse.to_dense() if sparse.is_sparse else sparse
    return grad_output @ dense_b.transpose(-1, -2), a.transpose(-1, -2) @ grad_output


def grad_fft1d(grad_output):
    """VJP of the unnormalised DFT along the last axis: the conjugate transform of the gradient."""
    return torch.fft.ifft(grad_output, dim=-1) * grad_output.shape[-1]
