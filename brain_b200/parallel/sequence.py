"""Sequence and context parallelism (absent in the reference; see the distributed component table).

* ``scatter_sequence`` / ``gather_sequence``: activations sharded along the sequence between tensor-
  parallel regions (SP), so norms and elementwise ops run on 1/world of the tokens.
* ``ring_attention``: context parallelism for long sequences. Each rank holds a contiguous sequence
  block of q/k/v; K/V blocks travel around the ring, each step computes attention of the local queries
  against the visiting block with the flash kernel (which returns the log-sum-exp), and partial
  results are merged with the online-softmax rule
      lse = logaddexp(lse_a, lse_b),  o = o_a * exp(lse_a - lse) + o_b * exp(lse_b - lse).
  Causal masking uses global positions: blocks entirely in the future are skipped, the diagonal
  block is causal, earlier blocks are full. (Forward / inference path; training uses SP + TP.)
* ``ulysses_attention``: all-to-all from sequence shards to head shards, local full attention,
  all-to-all back.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops


def scatter_sequence(x: torch.Tensor, rank: int, world: int, dim: int = 1) -> torch.Tensor:
    return torch.tensor_split(x, world, dim=dim)[rank].contiguous()


def gather_sequence(x: torch.Tensor, world: int, dim: int = 1, group=None) -> torch.Tensor:
    if world == 1:
        return x
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.cat(parts, dim=dim)


def _attn_with_lse(q, k, v, causal):
    if q.is_cuda:
        o, lse = ops.flash_attention_fwd(q, k, v, causal=causal)
        return o.float(), lse.transpose(1, 2)  # lse [B, Sq, H]
    import math
    D = q.shape[-1]
    rep = q.shape[2] // k.shape[2]
    qf, kf, vf = q.float().transpose(1, 2), k.float().transpose(1, 2).repeat_interleave(rep, 1), \
        v.float().transpose(1, 2).repeat_interleave(rep, 1)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(D)
    if causal:
        Sq, Sk = s.shape[-2:]
        i = torch.arange(Sq)[:, None]
        j = torch.arange(Sk)[None, :]
        s = s.masked_fill(j > i + (Sk - Sq), float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ vf
    return o.transpose(1, 2), lse.transpose(1, 2)


def merge_partials(o_a, lse_a, o_b, lse_b):
    lse = torch.logaddexp(lse_a, lse_b)
    wa = torch.exp(lse_a - lse).nan_to_num(0.0)[..., None]
    wb = torch.exp(lse_b - lse).nan_to_num(0.0)[..., None]
    return o_a * wa + o_b * wb, lse


def ring_attention(q, k, v, rank: int, world: int, causal: bool = True, group=None) -> torch.Tensor:
    """q/k/v: this rank's sequence block [B, S_local, H, D]; returns the local block of the output."""
    o_acc, lse_acc = None, None
    kk, vv = k.contiguous(), v.contiguous()
    for step in range(world):
        src = (rank - step) % world  # owner of the visiting K/V block
        if not causal or src <= rank:
            o, lse = _attn_with_lse(q, kk, vv, causal=(causal and src == rank))
            if o_acc is None:
                o_acc, lse_acc = o, lse
            else:
                o_acc, lse_acc = merge_partials(o_acc, lse_acc, o, lse)
        if step + 1 < world:
            nk, nv = torch.empty_like(kk), torch.empty_like(vv)
            right, left = (rank + 1) % world, (rank - 1) % world
            ops_ = [dist.P2POp(dist.isend, kk, right, group), dist.P2POp(dist.isend, vv, right, group),
                    dist.P2POp(dist.irecv, nk, left, group), dist.P2POp(dist.irecv, nv, left, group)]
            for w in dist.batch_isend_irecv(ops_):
                w.wait()
            kk, vv = nk, nv
    return o_acc.to(q.dtype)


def ulysses_attention(q, k, v, world: int, causal: bool = True, group=None) -> torch.Tensor:
    """Sequence-sharded [B, S/W, H, D] -> head-sharded full-sequence attention -> back."""
    def seq_to_head(x):
        B, s, H, D = x.shape
        x = x.reshape(B, s, world, H // world, D).permute(2, 0, 1, 3, 4).contiguous()
        out = torch.empty_like(x)
        dist.all_to_all_single(out, x, group=group)
        return out.permute(1, 0, 2, 3, 4).reshape(B, world * s, H // world, D)

    def head_to_seq(x, s):
        B, S, h, D = x.shape
        x = x.reshape(B, world, s, h, D).permute(1, 0, 2, 3, 4).contiguous()
        out = torch.empty_like(x)
        dist.all_to_all_single(out, x, group=group)
        return out.permute(1, 2, 0, 3, 4).reshape(B, s, world * h, D)

    s_local = q.shape[1]
    o = ops.flash_attention(seq_to_head(q), seq_to_head(k), seq_to_head(v), causal=causal)
    return head_to_seq(o, s_local)
