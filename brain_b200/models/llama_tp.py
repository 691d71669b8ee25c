"""Tensor-parallel Llama inference over the ranks of a process group (one GPU per rank).

Sharding (Megatron layout, head-aligned): rank r owns q heads [r*Hq/W, ...), kv heads [r*Hkv/W, ...),
FFN columns [r*F/W, ...) and vocabulary rows [r*ceil(V/W), ...); embeddings and norms are
replicated. Per layer the weights are ``wqkv`` [(Hq/W + 2 Hkv/W) * D, d] (this rank's q | k | v heads),
``wo`` [d, Hq/W * D], ``w_gu`` [2F/W, d] (gate and up rows interleaved in 64-row groups) and
``w_down`` [d, F/W].

Prefill (``prefill``): sequence parallel when the token count allows it - the residual stream is
sharded by tokens, QKV and gate/up run as all-gather -> GEMM pipelined by row block (copy-engine
pulls over NVLink overlapped with the GEMMs of blocks already present), out- and down-projections
as GEMM -> reduce-scatter (the epilogue pushes rows to their owners over NVLink); attention is the
tcgen05 flash-attention kernel over the local heads, and K/V land in the paged cache.

Decode (``step``; one token per sequence): every launch is a hand-written kernel and the whole step
is capturable as one CUDA graph (``capture``), because all per-step state (positions, sequence
lengths, all-reduce epochs) lives in device memory. Per layer:
  skinny GEMM + RoPE + KV-append (EPI_QKV) -> paged split-K decode attention -> skinny GEMM whose
  epilogue pushes its partial product to every rank (EPI_PUSH) -> all-reduce + residual + RMSNorm
  -> skinny GEMM + SwiGLU (EPI_SWIGLU) -> skinny GEMM push -> all-reduce + residual + RMSNorm;
then the vocabulary-parallel head with a fused greedy argmax whose keys are pushed to every rank,
and a pick kernel that records the token, advances the positions and embeds it for the next step.

Reference: LlamaLite::generate (crates/brain-transformer/src/llama_lite.rs) decodes greedily by
re-running the prefix; TensorParallelLinear (crates/brain-distributed/src/tensor_parallel.rs:8-27)
is a stub that returns zeros.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .. import ops
from ..ops.decode import (EPI_ARGMAX, EPI_PUSH, EPI_QKV, EPI_SWIGLU, ar_norm, decode_ext, decode_splits,
                          init_ar_slots, interleave_gate_up, paged_decode_attention, pick_embed, skinny_gemm,
                          skinny_splits)
from .config import LlamaLiteConfig


def _randn(shape, gen, std, device):
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


class _StepComm:
    """All-reduce and argmax-key receive slots of the decode step (symmetric when world > 1). Both are
    [2 parities][world][elems]; unwritten elements hold a sentinel that the consumers poll for."""

    def __init__(self, batch: int, hidden: int, world: int, rank: int, group, device):
        self.world, self.rank = world, rank
        self.ar_elems = batch * hidden
        self.key_elems = batch
        ar_bytes = 2 * world * self.ar_elems * 2
        key_bytes = 2 * world * self.key_elems * 8
        self.ar_off = 0
        self.key_off = -(-ar_bytes // 256) * 256
        total = self.key_off + key_bytes
        if world > 1:
            from ..parallel.symm import SymmetricBuffer
            self.buf = SymmetricBuffer(total, group)
            self.bases = list(self.buf.ptrs)
            self.local = self.buf.local
            self._keep = None
        else:
            self.buf = None
            self._keep = torch.zeros(total, device=device, dtype=torch.uint8)
            self.local = self._keep.data_ptr()
            self.bases = [self.local]
        self.ctrl = torch.zeros(4, device=device, dtype=torch.int32)  # epoch consumed, produced, ticket
        self.keys = torch.zeros(batch, device=device, dtype=torch.int64)
        self.ar_local = self.local + self.ar_off
        self.key_local = self.local + self.key_off
        slots = (self.buf.view(torch.bfloat16, 2 * world * self.ar_elems, self.ar_off) if self.buf is not None
                 else self._keep[self.ar_off:self.ar_off + ar_bytes].view(torch.bfloat16))
        init_ar_slots(slots)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier(group)  # every rank's slots hold the sentinel before any push

    def ext_push(self, l2_prefetch=None):
        return decode_ext(world=self.world, rank=self.rank, slot_elems=self.ar_elems, ctrl=self.ctrl,
                          peer_slots=[b + self.ar_off for b in self.bases], l2_prefetch=l2_prefetch)

    def ext_argmax(self, vocab_offset: int):
        return decode_ext(world=self.world, rank=self.rank, slot_elems=self.key_elems, ctrl=self.ctrl, keys=self.keys,
                          vocab_offset=vocab_offset, peer_slots=[b + self.key_off for b in self.bases])

    def close(self):
        if self.buf is not None:
            self.buf.close()
            self.buf = None


class LlamaTPServe:
    """Greedy batched generation of a Llama-shaped model, tensor-parallel over ``group``."""

    def __init__(self, cfg: LlamaLiteConfig, max_batch: int, max_len: int, block_size: int = 64, group=None,
                 seed: int = 0, init: bool = True, device=None, shard_of: int | None = None,
                 l2_prefetch: bool = False):
        """``shard_of`` (performance work on one GPU only): give this single rank the weight shard of one
        rank of a ``shard_of``-way group; the all-reduces then sum this shard alone, so the outputs are
        not the model's, but every kernel runs at the per-rank shapes of the larger group.
        ``l2_prefetch``: the decode step asks L2 for the small GEMMs' weights ahead of them (measured
        no faster on the 70B TP=8 shard step: 6.07 vs 6.04 ms, so off by default)."""
        self.cfg = cfg
        self.l2_prefetch = l2_prefetch
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if shard_of is not None and self.world != 1:
            raise ValueError("shard_of emulates a larger group on a single rank")
        W, c = (shard_of or self.world), cfg
        if c.num_heads % W or c.num_kv_heads % W or c.intermediate_dim % (64 * W):
            raise ValueError("heads, kv heads and FFN width / 64 must divide by the tensor-parallel size")
        if c.head_dim != 128:
            raise ValueError("the decode kernels are built for head_dim 128")
        if max_batch > 64:
            raise ValueError("decode batch is limited to 64 sequences per step")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        self.B, self.max_len, self.block_size = max_batch, max_len, block_size
        self.hq, self.hkv, self.D = c.num_heads // W, c.num_kv_heads // W, c.head_dim
        self.F = c.intermediate_dim // W
        self.V_shard = -(-c.vocab_size // W)
        self.v0 = self.rank * self.V_shard
        self.v_rows = max(0, min(self.V_shard, c.vocab_size - self.v0))
        d, L = c.hidden_dim, c.num_layers
        qkv_rows = (self.hq + 2 * self.hkv) * self.D
        # ---- weights
        self.emb = torch.empty(c.vocab_size, d, device=dev, dtype=torch.bfloat16)
        self.attn_norm = [torch.ones(d, device=dev, dtype=torch.bfloat16) for _ in range(L)]
        self.ffn_norm = [torch.ones(d, device=dev, dtype=torch.bfloat16) for _ in range(L)]
        self.final_norm = torch.ones(d, device=dev, dtype=torch.bfloat16)
        self.wqkv = [torch.empty(qkv_rows, d, device=dev, dtype=torch.bfloat16) for _ in range(L)]
        self.wo = [torch.empty(d, self.hq * self.D, device=dev, dtype=torch.bfloat16) for _ in range(L)]
        self.w_gu = [torch.empty(2 * self.F, d, device=dev, dtype=torch.bfloat16) for _ in range(L)]
        self.w_down = [torch.empty(d, self.F, device=dev, dtype=torch.bfloat16) for _ in range(L)]
        self.head = torch.empty(self.V_shard, d, device=dev, dtype=torch.bfloat16)
        if init:
            self._random_init(seed)
        # ---- paged KV cache: sequence b owns blocks [b * max_blocks, (b + 1) * max_blocks)
        self.max_blocks = -(-max_len // block_size)
        nblocks = max_batch * self.max_blocks
        self.kv = torch.empty(L, 2, nblocks, block_size, self.hkv, self.D, device=dev, dtype=torch.bfloat16)
        self.table = torch.arange(nblocks, device=dev, dtype=torch.int32).view(max_batch, self.max_blocks)
        self.rope = ops.rope_table(self.D, max_len, c.rope_theta, device=dev)
        # ---- decode state
        B = max_batch
        self.pos = torch.zeros(B, device=dev, dtype=torch.int32)
        self.seq_lens = torch.zeros(B, device=dev, dtype=torch.int32)
        self.hist = torch.zeros(B, max_len, device=dev, dtype=torch.int32)
        self.resid = torch.zeros(B, d, device=dev, dtype=torch.bfloat16)
        self.normed = torch.zeros(B, d, device=dev, dtype=torch.bfloat16)
        self.q = torch.empty(B, self.hq * self.D, device=dev, dtype=torch.bfloat16)
        self.attn = torch.empty(B, self.hq * self.D, device=dev, dtype=torch.bfloat16)
        self.act = torch.empty(B, self.F, device=dev, dtype=torch.bfloat16)
        self.attn_splits = decode_splits(B, self.hkv, self.D, max_len)
        self.comm = _StepComm(B, d, self.world, self.rank, group, dev)
        self.tp = None  # TPContext for the sequence-parallel prefill (created on first use)
        self.graph = None
        self._build_launch_args()

    # ------------------------------------------------------------------ weights
    def _random_init(self, seed: int):
        c, dev, std = self.cfg, self.device, self.cfg.init_std
        g_rep = torch.Generator(device=dev).manual_seed(seed)
        self.emb.copy_(_randn(self.emb.shape, g_rep, std, dev))
        g = torch.Generator(device=dev).manual_seed(seed * 7919 + 1 + self.rank)
        for layer in range(c.num_layers):
            for w in (self.wqkv[layer], self.wo[layer], self.w_gu[layer], self.w_down[layer]):
                w.copy_(_randn(w.shape, g, std, dev))
        self.head.zero_()
        self.head[:self.v_rows].copy_(_randn((self.v_rows, c.hidden_dim), g, std, dev))

    @torch.no_grad()
    def load_from(self, model) -> "LlamaTPServe":
        """Take this rank's shard of a ``LlamaLite`` (full weights on every rank)."""
        c, r, W = self.cfg, self.rank, self.world
        D, Hq, Hkv, F = self.D, c.num_heads, c.num_kv_heads, c.intermediate_dim
        self.emb.copy_(model.embed)
        for i, blk in enumerate(model.layers):
            self.attn_norm[i].copy_(blk.attn_norm)
            self.ffn_norm[i].copy_(blk.ffn_norm)
            w = blk.wqkv
            q = w[:Hq * D].view(Hq, D, -1)[r * self.hq:(r + 1) * self.hq]
            k = w[Hq * D:(Hq + Hkv) * D].view(Hkv, D, -1)[r * self.hkv:(r + 1) * self.hkv]
            v = w[(Hq + Hkv) * D:].view(Hkv, D, -1)[r * self.hkv:(r + 1) * self.hkv]
            self.wqkv[i].copy_(torch.cat([q, k, v], 0).reshape(-1, w.shape[1]))
            self.wo[i].copy_(blk.wo[:, r * self.hq * D:(r + 1) * self.hq * D])
            gate = blk.w_gate_up[:F][r * self.F:(r + 1) * self.F]
            up = blk.w_gate_up[F:][r * self.F:(r + 1) * self.F]
            self.w_gu[i].copy_(interleave_gate_up(gate, up))
            self.w_down[i].copy_(blk.w_down[:, r * self.F:(r + 1) * self.F])
        self.final_norm.copy_(model.final_norm)
        self.head.zero_()
        self.head[:self.v_rows].copy_(model.head_weight()[self.v0:self.v0 + self.v_rows])
        return self

    # ------------------------------------------------------------------ launch arguments
    def _build_launch_args(self):
        c, B, d = self.cfg, self.B, self.cfg.hidden_dim
        self.ext_qkv = [decode_ext(hq=self.hq, hkv=self.hkv, pos=self.pos, rope_cs=self.rope, k_pool=self.kv[i, 0],
                                   v_pool=self.kv[i, 1], block_table=self.table) for i in range(c.num_layers)]
        self.ext_push = self.comm.ext_push()
        # L2 prefetch of the small GEMMs' weights during the tails of the kernels before them: the decode
        # attention asks for this layer's out-projection, the down projection for the next layer's QKV
        self.ext_down = [self.comm.ext_push(l2_prefetch=self.wqkv[(i + 1) % c.num_layers] if self.l2_prefetch
                                            else None) for i in range(c.num_layers)]
        self.ext_argmax = self.comm.ext_argmax(self.v0)
        qkv_rows = self.wqkv[0].shape[0]
        self.sp = {
            "qkv": skinny_splits(B, qkv_rows, d), "o": skinny_splits(B, d, self.hq * self.D),
            "gu": skinny_splits(B, 2 * self.F, d), "down": skinny_splits(B, d, self.F),
            "head": skinny_splits(B, max(self.v_rows, 1), d),
        }
        self.gammas_after = [self.attn_norm[i + 1] for i in range(c.num_layers - 1)] + [self.final_norm]

    # ------------------------------------------------------------------ decode
    def _head_and_pick(self):
        c = self.cfg
        skinny_gemm(self.normed, self.head[:self.v_rows], EPI_ARGMAX, ext=self.ext_argmax, splits=self.sp["head"])
        cm = self.comm
        pick_embed(cm.key_local, cm.ctrl, self.world, cm.key_elems, self.emb, self.resid,
                   self.attn_norm[0], c.norm_eps, self.normed, self.hist, self.pos, self.seq_lens)

    def step(self):
        """One decode step for every sequence (eager launches; ``capture`` records the same launches)."""
        c, B, cm = self.cfg, self.B, self.comm
        for i in range(c.num_layers):
            skinny_gemm(self.normed, self.wqkv[i], EPI_QKV, out=self.q, ext=self.ext_qkv[i], splits=self.sp["qkv"])
            paged_decode_attention(self.q.view(B, self.hq, self.D), self.kv[i, 0], self.kv[i, 1], self.table,
                                   self.seq_lens, splits=self.attn_splits,
                                   l2_prefetch=self.wo[i] if self.l2_prefetch else None,
                                   out=self.attn.view(B, self.hq, self.D))
            skinny_gemm(self.attn, self.wo[i], EPI_PUSH, ext=self.ext_push, splits=self.sp["o"])
            ar_norm(cm.ar_local, cm.ctrl, self.world, cm.ar_elems, self.resid, self.ffn_norm[i],
                    c.norm_eps, self.normed)
            skinny_gemm(self.normed, self.w_gu[i], EPI_SWIGLU, out=self.act, splits=self.sp["gu"])
            skinny_gemm(self.act, self.w_down[i], EPI_PUSH, ext=self.ext_down[i], splits=self.sp["down"])
            ar_norm(cm.ar_local, cm.ctrl, self.world, cm.ar_elems, self.resid, self.gammas_after[i],
                    c.norm_eps, self.normed)
        self._head_and_pick()

    def launches_per_step(self) -> int:
        return self.cfg.num_layers * 7 + 2

    def capture(self):
        """Record one decode step as a CUDA graph (run ``prefill`` first: the kernels see real state)."""
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        self.graph = g
        return g

    def replay(self):
        self.graph.replay()

    # ------------------------------------------------------------------ prefill
    def _tp(self):
        if self.tp is None and self.world > 1:
            from ..parallel.tensor_parallel import TPContext
            self.tp = TPContext(self.group)
        return self.tp

    def _col(self, x, w, sp):
        """x [T_local or T, d] -> [T, n] with this rank's output columns."""
        if self.world > 1 and sp:
            from ..parallel.tensor_parallel import gemm_allgather_a
            return gemm_allgather_a(self._tp(), x, w)
        return ops.gemm(x, w, trans_b=True)

    def _row(self, x, w, sp, T):
        """Partial products of this rank's input columns, summed over ranks: [T/W, d] (sp) or [T, d]."""
        if self.world == 1:
            return ops.gemm(x, w, trans_b=True)
        from ..parallel.tensor_parallel import gemm_push
        return gemm_push(self._tp(), x.contiguous(), w, 1 if sp else 2, T // self.world if sp else T)

    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor) -> None:
        """Run the prompts tokens [B, S] (same length), fill the KV cache and pick the first new token."""
        c, W, D = self.cfg, self.world, self.D
        B, S = tokens.shape
        if B != self.B or S >= self.max_len:
            raise ValueError("prompt batch must equal max_batch and leave room to generate")
        T = B * S
        sp = W > 1 and T % W == 0 and (T // W) % 128 == 0
        rows = slice(self.rank * (T // W), (self.rank + 1) * (T // W)) if sp else slice(0, T)
        flat = tokens.reshape(-1).to(self.device, torch.int64)
        h = ops.embedding(flat[rows], self.emb).contiguous()
        xn = ops.rms_norm(h, self.attn_norm[0], c.norm_eps)
        for i in range(c.num_layers):
            qkv = self._col(xn, self.wqkv[i], sp).view(B, S, -1)
            o = ops.qkv_attention(qkv, self.hq, self.hkv, self.rope, causal=True)  # RoPE applied to qkv in place
            kvh = qkv.view(B, S, self.hq + 2 * self.hkv, D)
            pools = self.kv[i].view(2, B, self.max_blocks * self.block_size, self.hkv, D)
            pools[0, :, :S].copy_(kvh[:, :, self.hq:self.hq + self.hkv])
            pools[1, :, :S].copy_(kvh[:, :, self.hq + self.hkv:])
            a = self._row(o.reshape(T, -1), self.wo[i], sp, T)
            xn, h = ops.add_rms_norm(a, h, self.ffn_norm[i], c.norm_eps)
            gu = self._col(xn, self.w_gu[i], sp)
            act = ops.activations.swiglu_fwd_only(gu.view(-1, 128)).view(T, self.F)
            dn = self._row(act, self.w_down[i], sp, T)
            gamma = self.attn_norm[i + 1] if i + 1 < c.num_layers else self.final_norm
            xn, h = ops.add_rms_norm(dn, h, gamma, c.norm_eps)
        # last prompt token of every sequence -> decode state
        if sp:
            from ..parallel.tensor_parallel import all_gather_rows
            h = all_gather_rows(self._tp(), h)
            xn = all_gather_rows(self._tp(), xn)
        last = torch.arange(B, device=self.device) * S + (S - 1)
        self.resid.copy_(h[last])
        self.normed.copy_(xn[last])
        self.hist.zero_()
        self.hist[:, :S].copy_(tokens.to(self.device, torch.int32))
        self.pos.fill_(S - 1)
        self.seq_lens.fill_(S)
        self._head_and_pick()

    # ------------------------------------------------------------------ generation
    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, max_new_tokens: int, use_graph: bool = True) -> torch.Tensor:
        """Greedy continuation of prompt [B, S]; returns [B, S + max_new_tokens] (host int64)."""
        B, S = prompt.shape
        if S + max_new_tokens > self.max_len:
            raise ValueError("prompt + new tokens exceed max_len")
        self.prefill(prompt)
        steps = max_new_tokens - 1
        if steps > 0:
            self.step()  # eager first step (kernel attributes are set outside any capture)
            steps -= 1
        if use_graph and steps > 0 and self.graph is None:
            self.capture()  # records the launches without running them
        for _ in range(steps):
            if use_graph:
                self.replay()
            else:
                self.step()
        torch.cuda.synchronize()
        return self.hist[:, :S + max_new_tokens].to("cpu", torch.int64)

    def check(self) -> None:
        torch.cuda.synchronize()
        bad = ops.check_status()
        if bad:
            raise RuntimeError(f"decode kernels reported errors: {bad}")

    def close(self):
        self.graph = None
        torch.cuda.synchronize()
        self.comm.close()
        if self.tp is not None:
            self.tp.close()
            if self.tp.comm is not None:
                self.tp.comm.close()
            self.tp = None


def decode_bytes_per_step(cfg: LlamaLiteConfig, world: int, batch: int, avg_len: float) -> float:
    """HBM bytes one rank must read per decode step (weights once + its KV cache share)."""
    d, L, D = cfg.hidden_dim, cfg.num_layers, cfg.head_dim
    per_layer = ((cfg.num_heads + 2 * cfg.num_kv_heads) * D * d + d * cfg.num_heads * D
                 + 3 * d * cfg.intermediate_dim) / world
    weights = 2 * (L * per_layer + math.ceil(cfg.vocab_size / world) * d)
    kv = L * batch * avg_len * 2 * (cfg.num_kv_heads // world) * D * 2
    return weights + kv
