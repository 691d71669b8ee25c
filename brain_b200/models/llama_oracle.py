"""Float32 PyTorch restatement of one LlamaLite training step: the oracle for the fused kernels.

``loss_and_grads(model, tokens, labels)`` reads the weights of a :class:`LlamaLite` (any dtype, any
device), evaluates the same math with plain float32 torch ops and returns the mean next-token loss and
the gradient of every parameter by name. Nothing of the framework's kernels is on this path:
    h = embed[tokens]
    per block: qkv = rms(h) Wqkv^T, NeoX RoPE on the q and k heads, causal GQA softmax attention,
               h += o Wo^T;  gu = rms(h) Wgu^T;  h += (silu(gate) * up) Wdown^T
    loss = mean CE(rms(h) Whead^T, labels)
with the RoPE table of ``ops.rope_table`` (float64 angles rounded to float32) and RMSNorm
``x * rsqrt(mean(x^2) + eps) * w`` (crates/brain-transformer/src/ops.rs:103-131).

``adamw_reference(master, grad, ...)`` is one ``torch.optim.AdamW`` step in float32 on copies, used to
check the update the fused optimizer kernels apply.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x, table):
    # x [B, S, H, D]; table [>= S, D] float32: cos in [:, :D/2], sin in [:, D/2:]
    S, D = x.shape[1], x.shape[-1]
    half = D // 2
    c = table[:S, :half][None, :, None, :]
    s = table[:S, half:][None, :, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def _attention(q, k, v):
    # [B, S, H, D] with GQA; causal (square) in float32
    B, S, Hq, D = q.shape
    rep = Hq // k.shape[2]
    qt = q.transpose(1, 2)
    kt = k.transpose(1, 2).repeat_interleave(rep, dim=1)
    vt = v.transpose(1, 2).repeat_interleave(rep, dim=1)
    s = (qt @ kt.transpose(-1, -2)) / math.sqrt(D)
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    return (torch.softmax(s, dim=-1) @ vt).transpose(1, 2)


def loss_fp32(params: dict, cfg, tokens, labels, rope_table):
    """Mean CE of the LlamaLite forward on float32 ``params`` (name -> tensor)."""
    Hq, Hkv, hd, F_ = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.intermediate_dim
    h = params["embed"][tokens]
    for i in range(cfg.num_layers):
        p = lambda n: params[f"layers.{i}.{n}"]  # noqa: E731
        B, S, _ = h.shape
        qkv = (_rms(h, p("attn_norm"), cfg.norm_eps) @ p("wqkv").t()).view(B, S, Hq + 2 * Hkv, hd)
        q, k, v = qkv.split([Hq, Hkv, Hkv], dim=2)
        o = _attention(_rope(q, rope_table), _rope(k, rope_table), v).reshape(B, S, Hq * hd)
        h = h + o @ p("wo").t()
        gu = _rms(h, p("ffn_norm"), cfg.norm_eps) @ p("w_gate_up").t()
        h = h + (F.silu(gu[..., :F_]) * gu[..., F_:]) @ p("w_down").t()
    head = params["embed"] if cfg.tie_embeddings else params["lm_head"]
    logits = _rms(h, params["final_norm"], cfg.norm_eps) @ head.t()
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels.reshape(-1))


def loss_and_grads(model, tokens, labels, device=None):
    """(loss, {name: grad}) of ``model``'s weights in float32 (on ``device``, default the model's)."""
    from ..ops.rope import rope_table
    cfg = model.config
    dev = device or next(model.parameters()).device
    params = {n: p.detach().to(dev, torch.float32).clone().requires_grad_(True) for n, p in model.named_parameters()}
    table = rope_table(cfg.head_dim, tokens.shape[1], cfg.rope_theta, device=dev)
    loss = loss_fp32(params, cfg, tokens.to(dev), labels.to(dev), table)
    loss.backward()
    return loss.detach(), {n: p.grad for n, p in params.items()}


def adamw_reference(master: torch.Tensor, grads: list[torch.Tensor], lr: float, betas=(0.9, 0.999), eps: float = 1e-8,
                    weight_decay: float = 0.0) -> torch.Tensor:
    """Weights after ``len(grads)`` steps of ``torch.optim.AdamW`` (float32) from ``master``."""
    w = torch.nn.Parameter(master.detach().float().clone())
    opt = torch.optim.AdamW([w], lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, foreach=False)
    for g in grads:
        w.grad = g.detach().float().to(w.device)
        opt.step()
    return w.detach()


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b|| in float64."""
    a, b = a.double(), b.double().to(a.device)
    return float((a - b).norm() / b.norm().clamp_min(1e-30))
