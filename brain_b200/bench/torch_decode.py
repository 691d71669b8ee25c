"""Plain-PyTorch baseline of the tensor-parallel decode benchmark: the Llama-3-70B-shaped model served
with eager torch ops and nothing from this framework.

Each rank holds a Megatron-style shard: the QKV and gate/up projections split by output (heads and
FFN columns), the output and down projections split by input and summed with
``torch.distributed.all_reduce`` over NCCL, the LM head split by vocabulary with the greedy pick taken
over an all-gather of every rank's (max, argmax). GEMMs are ``F.linear`` (cuBLAS), attention is
``F.scaled_dot_product_attention`` over a contiguous per-layer KV cache, RMSNorm is ``F.rms_norm``,
RoPE and SwiGLU are torch elementwise ops.

The decode step is written with static shapes (the cache is read to its full capacity under an
additive mask, the position lives in a device tensor) so that it can be captured once in a CUDA
graph and replayed, the way a PyTorch server removes launch overhead; ``graph=False`` runs it
eagerly. ``shard_of=N`` on one process builds one rank's shard of an N-way group and skips the
collectives (a single-GPU view of the per-rank work).

Reference semantics (greedy next token from the last position, RoPE, GQA, SwiGLU, RMSNorm):
``crates/brain-transformer/src/models/llama.rs`` forward and ``generation/mod.rs`` greedy decoding.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn.functional as F


class TorchTPDecoder:
    def __init__(self, cfg, max_batch: int, max_len: int, device, world: int = 1, rank: int = 0,
                 shard_of: int | None = None, seed: int = 0, group=None, dtype=torch.bfloat16):
        self.cfg, self.dev = cfg, torch.device(device)
        self.tp = shard_of or world
        self.collective = shard_of is None and world > 1
        self.group = group
        tp = self.tp
        if cfg.num_heads % tp or cfg.num_kv_heads % tp or cfg.intermediate_dim % tp or cfg.vocab_size % tp:
            raise ValueError(f"model does not split {tp} ways")
        self.hq, self.hkv, self.hd = cfg.num_heads // tp, cfg.num_kv_heads // tp, cfg.head_dim
        self.ffn, self.vloc = cfg.intermediate_dim // tp, cfg.vocab_size // tp
        self.B, self.T = max_batch, max_len
        d = cfg.hidden_dim
        g = torch.Generator(device=self.dev).manual_seed(seed * 1000 + rank)
        bf = dtype

        def w(*shape):
            return (torch.randn(*shape, device=self.dev, generator=g) * 0.02).to(bf)

        self.embed = w(cfg.vocab_size, d)  # replicated
        self.layers = []
        for _ in range(cfg.num_layers):
            self.layers.append({
                "wqkv": w((self.hq + 2 * self.hkv) * self.hd, d), "wo": w(d, self.hq * self.hd),
                "wgu": w(2 * self.ffn, d), "wd": w(d, self.ffn),
                "n1": torch.ones(d, device=self.dev, dtype=bf), "n2": torch.ones(d, device=self.dev, dtype=bf)})
        self.norm = torch.ones(d, device=self.dev, dtype=bf)
        self.head = w(self.vloc, d)
        L = cfg.num_layers
        self.kc = torch.zeros(L, max_batch, self.hkv, max_len, self.hd, device=self.dev, dtype=bf)
        self.vc = torch.zeros_like(self.kc)
        inv = 1.0 / cfg.rope_theta ** (torch.arange(0, self.hd, 2, device=self.dev, dtype=torch.float32) / self.hd)
        ang = torch.outer(torch.arange(max_len, device=self.dev, dtype=torch.float32), inv)
        ang = torch.cat([ang, ang], dim=-1)
        self.cos, self.sin = ang.cos().to(bf), ang.sin().to(bf)
        self.pos = torch.zeros((), device=self.dev, dtype=torch.long)  # next position to write
        self.tok = torch.zeros(max_batch, device=self.dev, dtype=torch.long)  # current input tokens
        self.graph = None
        self.rank = rank

    # ------------------------------------------------------------------ pieces
    def _allreduce(self, x):
        if self.collective:
            dist.all_reduce(x, group=self.group)
        return x

    @staticmethod
    def _rope(x, cos, sin):
        half = x.shape[-1] // 2
        return x * cos + torch.cat([-x[..., half:], x[..., :half]], dim=-1) * sin

    def _mlp(self, lw, x):
        h = F.rms_norm(x, (x.shape[-1],), lw["n2"], self.cfg.norm_eps)
        gt, up = F.linear(h, lw["wgu"]).chunk(2, dim=-1)
        return x + self._allreduce(F.linear(F.silu(gt) * up, lw["wd"]))

    def _greedy(self, h):
        """Global argmax over the vocabulary-sharded logits of h [B, d]."""
        logits = F.linear(F.rms_norm(h, (h.shape[-1],), self.norm, self.cfg.norm_eps), self.head).float()
        val, idx = logits.max(dim=-1)
        if not self.collective:
            return idx + self.rank * self.vloc if self.tp == 1 else idx
        both = torch.stack([val, (idx + self.rank * self.vloc).float()], dim=0)  # [2, B]
        outs = torch.empty(dist.get_world_size(self.group), 2, h.shape[0], device=self.dev)
        dist.all_gather_into_tensor(outs, both, group=self.group)
        best = outs[:, 0].argmax(dim=0)  # lowest rank wins ties, as the lowest vocabulary index would
        return outs[:, 1].gather(0, best[None]).squeeze(0).long()

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, prompts: torch.Tensor, chunk: int = 4) -> torch.Tensor:
        """Run the prompts [B, S] (all the same length), fill the caches, return the first new tokens."""
        B, S = prompts.shape
        cos, sin = self.cos[:S], self.sin[:S]
        nxt = torch.empty(B, device=self.dev, dtype=torch.long)
        for b0 in range(0, B, chunk):
            b1 = min(B, b0 + chunk)
            x = self.embed[prompts[b0:b1]]
            for li, lw in enumerate(self.layers):
                h = F.rms_norm(x, (x.shape[-1],), lw["n1"], self.cfg.norm_eps)
                qkv = F.linear(h, lw["wqkv"]).view(b1 - b0, S, self.hq + 2 * self.hkv, self.hd).transpose(1, 2)
                q, k, v = qkv.split([self.hq, self.hkv, self.hkv], dim=1)
                q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
                self.kc[li, b0:b1, :, :S] = k
                self.vc[li, b0:b1, :, :S] = v
                o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
                x = x + self._allreduce(F.linear(o.transpose(1, 2).reshape(b1 - b0, S, -1), lw["wo"]))
                x = self._mlp(lw, x)
            nxt[b0:b1] = self._greedy(x[:, -1])
        self.pos.fill_(S)
        self.tok.copy_(nxt)
        return nxt

    # ------------------------------------------------------------------ decode
    @torch.no_grad()
    def _step(self) -> None:
        """One token for every sequence at position self.pos (static shapes: graph-capturable)."""
        B, T = self.B, self.T
        pos = self.pos
        cos, sin = self.cos.index_select(0, pos[None]), self.sin.index_select(0, pos[None])
        # additive mask over the whole cache capacity: keys at or before pos are visible
        mask = torch.where(torch.arange(T, device=self.dev) <= pos, 0.0, -math.inf).to(self.kc.dtype)
        mask = mask.view(1, 1, 1, T)
        g = self.hq // self.hkv
        x = self.embed[self.tok][:, None]  # [B, 1, d]
        for li, lw in enumerate(self.layers):
            h = F.rms_norm(x, (x.shape[-1],), lw["n1"], self.cfg.norm_eps)
            qkv = F.linear(h, lw["wqkv"]).view(B, 1, self.hq + 2 * self.hkv, self.hd).transpose(1, 2)
            q, k, v = qkv.split([self.hq, self.hkv, self.hkv], dim=1)
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            self.kc[li].index_copy_(2, pos[None], k)
            self.vc[li].index_copy_(2, pos[None], v)
            # one query per sequence: the g query heads of a KV head attend as g query rows of that head
            o = F.scaled_dot_product_attention(q.reshape(B, self.hkv, g, self.hd), self.kc[li], self.vc[li],
                                               attn_mask=mask)
            x = x + self._allreduce(F.linear(o.reshape(B, 1, -1), lw["wo"]))
            x = self._mlp(lw, x)
        self.tok.copy_(self._greedy(x[:, 0]))
        self.pos.add_(1)

    def capture(self) -> None:
        """Capture one decode step in a CUDA graph (after at least one eager step has warmed it up)."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        pos0, tok0 = self.pos.clone(), self.tok.clone()
        with torch.cuda.stream(s):
            self._step()  # side-stream warm-up, required before capture with NCCL and cuBLAS workspaces
        torch.cuda.current_stream().wait_stream(s)
        self.pos.copy_(pos0)
        self.tok.copy_(tok0)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        # capture recorded the work without running it: the state is still at pos0

    def step(self, graph: bool = True) -> torch.Tensor:
        if graph and self.graph is not None:
            self.graph.replay()
        else:
            self._step()
        return self.tok

    @torch.no_grad()
    def generate(self, prompts: torch.Tensor, new_tokens: int, graph: bool = True) -> torch.Tensor:
        """Greedy generation: prefill, then new_tokens - 1 decode steps; returns [B, S + new_tokens]."""
        B, S = prompts.shape
        out = torch.empty(B, S + new_tokens, device=self.dev, dtype=torch.long)
        out[:, :S] = prompts
        out[:, S] = self.prefill(prompts)
        for i in range(1, new_tokens):
            out[:, S + i] = self.step(graph)
        return out

    def close(self) -> None:
        self.graph = None  # a graph holding NCCL calls goes before the process group
