"""Data pipeline (crates/brain-data, crates/brain-dataset): samplers (including the disjoint per-replica
``DistributedSampler``, brain-data/src/samplers.rs:37), datasets, a ``DataLoader`` with pinned-memory
batches and background prefetch, memory-mapped token streams, and the seeded synthetic generators
used by the benchmarks (uniform tokens, N(0,1) images)."""
from __future__ import annotations

import math
import os
import queue
import threading

import numpy as np
import torch


class Dataset:
    def __len__(self):  # pragma: no cover - abstract
        raise NotImplementedError

    def __getitem__(self, i):  # pragma: no cover - abstract
        raise NotImplementedError


class TensorDataset(Dataset):
    def __init__(self, *tensors):
        assert all(len(t) == len(tensors[0]) for t in tensors)
        self.tensors = tensors

    def __len__(self):
        return len(self.tensors[0])

    def __getitem__(self, i):
        return tuple(t[i] for t in self.tensors)


class SyntheticTokens(Dataset):
    """Uniform random token sequences of length seq+1 (inputs + shifted labels), seeded per index."""

    def __init__(self, vocab_size: int, seq_len: int, num_samples: int, seed: int = 1):
        self.v, self.s, self.n, self.seed = vocab_size, seq_len, num_samples, seed

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + i)
        t = torch.randint(0, self.v, (self.s + 1,), generator=g)
        return t[:-1], t[1:]


class SyntheticImages(Dataset):
    """N(0,1) images [C, H, W] with uniform labels (the ViT benchmark data)."""

    def __init__(self, num_samples: int, image_size=224, channels=3, num_classes=1000, seed: int = 0):
        self.n, self.hw, self.c, self.k, self.seed = num_samples, image_size, channels, num_classes, seed

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + i)
        return torch.randn(self.c, self.hw, self.hw, generator=g), int(torch.randint(self.k, (1,), generator=g))


class MmapTokens(Dataset):
    """Fixed-length windows over a flat token file (uint16 / uint32 / int32), memory mapped."""

    def __init__(self, path: str, seq_len: int, dtype=np.uint16):
        self.data = np.memmap(path, dtype=dtype, mode="r")
        self.s = seq_len

    def __len__(self):
        return max(0, (len(self.data) - 1) // self.s)

    def __getitem__(self, i):
        w = torch.from_numpy(self.data[i * self.s: i * self.s + self.s + 1].astype(np.int64))
        return w[:-1], w[1:]


class SequentialSampler:
    def __init__(self, n: int):
        self.n = n

    def __iter__(self):
        return iter(range(self.n))

    def __len__(self):
        return self.n


class RandomSampler(SequentialSampler):
    def __init__(self, n: int, seed: int = 0):
        super().__init__(n)
        self.seed, self.epoch = seed, 0

    def set_epoch(self, e: int):
        self.epoch = e

    def __iter__(self):
        g = torch.Generator().manual_seed(self.seed + self.epoch)
        return iter(torch.randperm(self.n, generator=g).tolist())


class DistributedSampler(RandomSampler):
    """Disjoint, equally sized per-replica index sets (padded by wrapping)."""

    def __init__(self, n: int, num_replicas: int, rank: int, shuffle: bool = True, seed: int = 0,
                 drop_last: bool = False):
        super().__init__(n, seed)
        self.replicas, self.rank, self.shuffle, self.drop_last = num_replicas, rank, shuffle, drop_last
        self.per = n // num_replicas if drop_last else math.ceil(n / num_replicas)

    def __iter__(self):
        idx = list(super().__iter__()) if self.shuffle else list(range(self.n))
        total = self.per * self.replicas
        if self.drop_last:
            idx = idx[:total]
        else:
            idx = (idx * math.ceil(total / max(1, len(idx))))[:total]
        return iter(idx[self.rank:total:self.replicas])

    def __len__(self):
        return self.per


def default_collate(items):
    first = items[0]
    if isinstance(first, tuple):
        return tuple(default_collate([it[k] for it in items]) for k in range(len(first)))
    if isinstance(first, torch.Tensor):
        return torch.stack(items)
    return torch.tensor(items)


class DataLoader:
    """Batches from a dataset + sampler; optional pinned memory and a background prefetch thread."""

    def __init__(self, dataset, batch_size=1, sampler=None, shuffle=False, drop_last=False, collate=default_collate,
                 pin_memory=False, prefetch: int = 2, seed: int = 0):
        self.ds, self.bs, self.drop_last, self.collate = dataset, batch_size, drop_last, collate
        self.sampler = sampler or (RandomSampler(len(dataset), seed) if shuffle else SequentialSampler(len(dataset)))
        self.pin = pin_memory and torch.cuda.is_available()
        self.prefetch = prefetch

    def _batches(self):
        buf = []
        for i in self.sampler:
            buf.append(self.ds[i])
            if len(buf) == self.bs:
                yield self._finish(buf)
                buf = []
        if buf and not self.drop_last:
            yield self._finish(buf)

    def _finish(self, buf):
        b = self.collate(buf)
        if self.pin:
            b = tuple(t.pin_memory() for t in b) if isinstance(b, tuple) else b.pin_memory()
        return b

    def __iter__(self):
        if self.prefetch <= 0:
            yield from self._batches()
            return
        q: queue.Queue = queue.Queue(self.prefetch)
        done = object()

        def work():
            try:
                for b in self._batches():
                    q.put(b)
            finally:
                q.put(done)
        t = threading.Thread(target=work, daemon=True)
        t.start()
        while True:
            b = q.get()
            if b is done:
                break
            yield b

    def __len__(self):
        n = len(self.sampler)
        return n // self.bs if self.drop_last else math.ceil(n / self.bs)


def random_split(n: int, fractions, seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n, generator=g).tolist()
    out, start = [], 0
    for i, f in enumerate(fractions):
        k = n - start if i == len(fractions) - 1 else int(round(f * n))
        out.append(perm[start:start + k])
        start += k
    return out


def write_token_file(path: str, tokens, dtype=np.uint16) -> None:
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    np.asarray(tokens, dtype=dtype).tofile(path)
