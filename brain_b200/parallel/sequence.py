"""Sequence and context parallelism (absent in the reference; see the distributed component table).

* ``scatter_sequence`` / ``gather_sequence``: activations sharded along the sequence between tensor-
  parallel regions (SP), so norms and elementwise ops run on 1/world of the tokens.
* ``ring_attention``: context parallelism for long sequences. Each rank holds a contiguous sequence
  block of q/k/v; K/V blocks travel around the ring, each step computes attention of the local queries
  against the visiting block with the flash kernel (which returns the log-sum-exp), and partial
  results are merged with the online-softmax rule
      lse = logaddexp(lse_a, lse_b),  o = o_a * exp(lse_a - lse) + o_b * exp(lse_b - lse).
  Causal masking uses global positions: blocks entirely in the future are skipped, the diagonal
  block is causal, earlier blocks are full. The next block's transfer is posted before the current
  block's attention runs, so it overlaps the compute. ``ring_attention`` is differentiable: the backward
  visits the blocks again and runs the flash backward of each (q, K_j, V_j) pair against the final
  (o, lse), which gives exactly that block's share of dq, dk, dv; the dK/dV accumulators travel with
  their K/V block and arrive back at its owner after the last hop.
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


def _ring_shift(tensors, rank, world, group):
    """Post sends of ``tensors`` to rank+1 and receives of same-shaped buffers from rank-1; returns
    (received buffers, works)."""
    right, left = (rank + 1) % world, (rank - 1) % world
    recv = [torch.empty_like(t) for t in tensors]
    ops_ = [dist.P2POp(dist.isend, t, right, group) for t in tensors] + \
           [dist.P2POp(dist.irecv, r, left, group) for r in recv]
    return recv, dist.batch_isend_irecv(ops_)


def _block_bwd_ref(q, k, v, o, lse, do, causal, scale):
    """float32 gradient shares of one (q, K_j, V_j) block given the final o and lse [B, Sq, H]."""
    rep = q.shape[2] // k.shape[2]
    qf, of, dof = (x.float().transpose(1, 2) for x in (q, o, do))
    kf = k.float().transpose(1, 2).repeat_interleave(rep, 1)
    vf = v.float().transpose(1, 2).repeat_interleave(rep, 1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        Sq, Sk = s.shape[-2:]
        i = torch.arange(Sq)[:, None]
        j = torch.arange(Sk)[None, :]
        s = s.masked_fill(j > i + (Sk - Sq), float("-inf"))
    p = torch.exp(s - lse.transpose(1, 2)[..., None].float())
    dv = p.transpose(-1, -2) @ dof
    dp = dof @ vf.transpose(-1, -2)
    delta = (dof * of).sum(-1, keepdim=True)
    ds = p * (dp - delta)
    dq = (ds @ kf) * scale
    dk = (ds.transpose(-1, -2) @ qf) * scale
    B, H, Sk, D = dk.shape
    dk = dk.view(B, H // rep, rep, Sk, D).sum(2)
    dv = dv.view(B, H // rep, rep, Sk, D).sum(2)
    return dq.transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2)


class _RingAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, rank, world, causal, group):
        o_acc, lse_acc = None, None
        kk, vv = k.contiguous(), v.contiguous()
        for step in range(world):
            src = (rank - step) % world  # owner of the visiting K/V block
            nxt = _ring_shift([kk, vv], rank, world, group) if step + 1 < world else None
            if not causal or src <= rank:
                o, lse = _attn_with_lse(q, kk, vv, causal=(causal and src == rank))
                if o_acc is None:
                    o_acc, lse_acc = o, lse
                else:
                    o_acc, lse_acc = merge_partials(o_acc, lse_acc, o, lse)
            if nxt is not None:
                (kk, vv), works = nxt
                for w in works:
                    w.wait()
        out = o_acc.to(q.dtype)
        ctx.save_for_backward(q, k, v, out, lse_acc.contiguous())
        ctx.meta = (rank, world, causal, group)
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        rank, world, causal, group = ctx.meta
        import math
        scale = 1.0 / math.sqrt(q.shape[-1])
        do = do.contiguous()
        dq = torch.zeros(q.shape, device=q.device, dtype=torch.float32)
        kk, vv = k.contiguous(), v.contiguous()
        dkk = torch.zeros(k.shape, device=k.device, dtype=torch.float32)
        dvv = torch.zeros(v.shape, device=v.device, dtype=torch.float32)
        lse_bhs = lse.transpose(1, 2).contiguous()  # the kernels' [B, H, S] layout
        for step in range(world):
            src = (rank - step) % world
            # K/V move on ahead of their gradient accumulators: post their transfer before the compute
            nxt = _ring_shift([kk, vv], rank, world, group) if step + 1 < world else None
            if not causal or src <= rank:
                blk_causal = causal and src == rank
                if q.is_cuda:
                    from ..ops import attention as attn
                    dq_j, dk_j, dv_j = torch.empty_like(q), torch.empty_like(kk), torch.empty_like(vv)
                    attn._bwd(q, kk, vv, o, lse_bhs, do, dq_j, dk_j, dv_j, blk_causal, scale)
                else:
                    dq_j, dk_j, dv_j = _block_bwd_ref(q, kk, vv, o, lse, do, blk_causal, scale)
                dq += dq_j.float()
                dkk += dk_j.float()
                dvv += dv_j.float()
            if nxt is not None:
                (kk, vv), works = nxt
                (dkk, dvv), works2 = _ring_shift([dkk, dvv], rank, world, group)
                for w in works + works2:
                    w.wait()
        # after world - 1 hops the accumulators sit one rank ahead of their owner: one more hop home
        if world > 1:
            (dkk, dvv), works = _ring_shift([dkk, dvv], rank, world, group)
            for w in works:
                w.wait()
        return dq.to(q.dtype), dkk.to(k.dtype), dvv.to(v.dtype), None, None, None, None


def ring_attention(q, k, v, rank: int, world: int, causal: bool = True, group=None) -> torch.Tensor:
    """q/k/v: this rank's sequence block [B, S_local, H, D] (block ``rank`` of the sequence, GQA allowed);
    returns the local block of the output. Differentiable (context-parallel training)."""
    return _RingAttentionFn.apply(q, k, v, rank, world, causal, group)


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
