"""KV caches for incremental decoding.

``KvCache`` keeps the reference API (``KvCache::new(KvCacheConfig)``, ``update(layer, k, v) ->
(full_k, full_v)``, ``clear``, ``current_seq_len``; crates/brain-transformer/src/kv_cache.rs:45-220)
but never reallocates: each layer owns a preallocated ``[B, max_len, Hkv, D]`` buffer, ``update``
writes the new positions in place and returns strided views that the attention kernel reads
directly (the reference copies the whole cache on every append).

``PagedKvCache`` stores K/V in fixed-size blocks ``[num_blocks, block_size, Hkv, D]`` addressed by
per-sequence block tables, for serving many sequences of different lengths; the paged decode
kernel (``ops.paged_decode_attention``) reads it without gathering.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class KvCacheConfig:
    num_layers: int
    batch_size: int
    num_kv_heads: int
    head_dim: int
    max_seq_len: int
    dtype: torch.dtype = torch.bfloat16
    device: str | torch.device = "cuda"


class KvCache:
    def __init__(self, config: KvCacheConfig):
        self.config = config
        c = config
        shape = (c.batch_size, c.max_seq_len, c.num_kv_heads, c.head_dim)
        self.k = [torch.empty(shape, dtype=c.dtype, device=c.device) for _ in range(c.num_layers)]
        self.v = [torch.empty(shape, dtype=c.dtype, device=c.device) for _ in range(c.num_layers)]
        self.lengths = [0] * c.num_layers

    def update(self, layer: int, k: torch.Tensor, v: torch.Tensor):
        """Append k/v [B, s, Hkv, D] for `layer`; returns views of the whole cached sequence."""
        t0 = self.lengths[layer]
        s = k.shape[1]
        if t0 + s > self.config.max_seq_len:
            raise ValueError(f"KV cache overflow: {t0 + s} > max_seq_len {self.config.max_seq_len}")
        self.k[layer][:, t0:t0 + s].copy_(k)
        self.v[layer][:, t0:t0 + s].copy_(v)
        self.lengths[layer] = t0 + s
        return self.k[layer][:, :t0 + s], self.v[layer][:, :t0 + s]

    def current_seq_len(self, layer: int = 0) -> int:
        return self.lengths[layer]

    def clear(self):
        self.lengths = [0] * self.config.num_layers

    def memory_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)


class PagedKvCache:
    """Block-paged cache: per layer K/V pools [num_blocks, block_size, Hkv, D] + block tables."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                 dtype=torch.bfloat16, device="cuda"):
        self.num_layers, self.block_size = num_layers, block_size
        shape = (num_blocks, block_size, num_kv_heads, head_dim)
        self.k = [torch.empty(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.v = [torch.empty(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.free = list(range(num_blocks - 1, -1, -1))
        self.tables: dict[int, list[int]] = {}
        self.seq_lens: dict[int, int] = {}
        self.device = device

    def add_sequence(self, seq_id: int) -> None:
        self.tables[seq_id] = []
        self.seq_lens[seq_id] = 0

    def free_sequence(self, seq_id: int) -> None:
        self.free.extend(reversed(self.tables.pop(seq_id)))
        self.seq_lens.pop(seq_id)

    def reserve(self, seq_id: int, new_tokens: int) -> None:
        need = -(-(self.seq_lens[seq_id] + new_tokens) // self.block_size)
        tab = self.tables[seq_id]
        while len(tab) < need:
            if not self.free:
                raise RuntimeError("paged KV cache out of blocks")
            tab.append(self.free.pop())

    def slot_mapping(self, seq_ids: list[int], new_tokens: int) -> torch.Tensor:
        """Flat slot (block * block_size + offset) of each new token, [len(seq_ids) * new_tokens]."""
        slots = []
        for sid in seq_ids:
            base = self.seq_lens[sid]
            tab = self.tables[sid]
            for t in range(base, base + new_tokens):
                slots.append(tab[t // self.block_size] * self.block_size + t % self.block_size)
        return torch.tensor(slots, dtype=torch.int64, device=self.device)

    def advance(self, seq_ids: list[int], new_tokens: int) -> None:
        for sid in seq_ids:
            self.seq_lens[sid] += new_tokens

    def block_table_tensor(self, seq_ids: list[int]) -> torch.Tensor:
        width = max(len(self.tables[s]) for s in seq_ids)
        out = torch.zeros(len(seq_ids), width, dtype=torch.int32)
        for i, s in enumerate(seq_ids):
            out[i, :len(self.tables[s])] = torch.tensor(self.tables[s], dtype=torch.int32)
        return out.to(self.device)

    def lengths_tensor(self, seq_ids: list[int]) -> torch.Tensor:
        return torch.tensor([self.seq_lens[s] for s in seq_ids], dtype=torch.int32, device=self.device)

    def write(self, layer: int, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        """Scatter new k/v [n, Hkv, D] into their slots."""
        kp = self.k[layer].view(-1, *self.k[layer].shape[2:])
        vp = self.v[layer].view(-1, *self.v[layer].shape[2:])
        kp.index_copy_(0, slots, k.reshape(-1, *kp.shape[1:]))
        vp.index_copy_(0, slots, v.reshape(-1, *vp.shape[1:]))

    def gather(self, layer: int, seq_id: int):
        """Contiguous [T, Hkv, D] copies of one sequence (testing / fallback)."""
        T = self.seq_lens[seq_id]
        idx = torch.tensor(self.tables[seq_id], device=self.device, dtype=torch.long)
        k = self.k[layer][idx].reshape(-1, *self.k[layer].shape[2:])[:T]
        v = self.v[layer][idx].reshape(-1, *self.v[layer].shape[2:])[:T]
        return k, v
