"""Data-pipeline stages with the reference's names: ``PrefetchIter`` (a background producer behind a
bounded queue: back-pressure when the consumer is slow), ``MapStage`` / ``PipelineRunner`` (a chain of
per-batch transforms with per-stage timing in ``StageProfile``), ``MemoryLoader`` (in-memory tensors in
batches), ``LazySample``, ``ConcatSources``, seeded ``shuffle_indices``, ``pad_and_stack_sequences``,
``stack_samples_to_tensor``, ``dedup_items`` and ``fnv_hash_bytes``; synthetic image, segmentation and
audio datasets.

Reference: crates/brain-data/src/prefetch.rs (PrefetchIter::from_iterator / from_batches_bounded),
stages.rs (MapStage), impl.rs (PipelineRunner::run_epoch), profile.rs (StageProfile), loading.rs
(MemoryLoader::from_tensors), lazy.rs, multi.rs (ConcatSources), shuffle.rs, collate.rs, utils.rs
(dedup_items, fnv_hash_bytes: 64-bit FNV-1a); crates/brain-dataset/src/dataset/{vision,vision_v2,audio}.rs.
"""
from __future__ import annotations

import queue
import threading
import time
from dataclasses import dataclass, field

import torch

from . import ConcatDataset, Dataset

ConcatSources = ConcatDataset

_FNV_OFFSET, _FNV_PRIME = 0xCBF29CE484222325, 0x100000001B3


def fnv_hash_bytes(data: bytes) -> int:
    """64-bit FNV-1a."""
    h = _FNV_OFFSET
    for b in data:
        h = ((h ^ b) * _FNV_PRIME) & 0xFFFFFFFFFFFFFFFF
    return h


def dedup_items(items, key=None) -> list:
    """Items in first-seen order without repeats (by ``key(item)`` when given)."""
    seen, out = set(), []
    for it in items:
        k = key(it) if key else it
        if k not in seen:
            seen.add(k)
            out.append(it)
    return out


def shuffle_indices(n: int, seed: int) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(n, generator=g).tolist()


def pad_and_stack_sequences(seqs, pad_value=0, max_len: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Variable-length [L_i, ...] tensors -> ([B, L, ...] padded, lengths [B])."""
    seqs = [torch.as_tensor(s) for s in seqs]
    lens = torch.tensor([s.shape[0] for s in seqs])
    L = max_len if max_len is not None else int(lens.max()) if len(seqs) else 0
    out = torch.full((len(seqs), L, *seqs[0].shape[1:]), pad_value, dtype=seqs[0].dtype) if seqs else torch.empty(0)
    for i, s in enumerate(seqs):
        n = min(L, s.shape[0])
        out[i, :n] = s[:n]
    return out, lens.clamp(max=L)


def stack_samples_to_tensor(samples) -> torch.Tensor:
    return torch.stack([torch.as_tensor(s) for s in samples])


class LazySample:
    """A sample computed on first access and cached."""

    def __init__(self, fn):
        self._fn, self._done, self._v = fn, False, None

    def get(self):
        if not self._done:
            self._v, self._done = self._fn(), True
        return self._v

    @property
    def is_loaded(self) -> bool:
        return self._done


class PrefetchIter:
    """Runs the source iterator in a daemon thread, ``capacity`` items ahead. The producer blocks when
    the queue is full (back-pressure); an exception in the producer is re-raised in the consumer."""

    _END = object()

    def __init__(self, source, capacity: int = 4):
        self._q: queue.Queue = queue.Queue(maxsize=max(1, capacity))
        self._stop = threading.Event()
        self.produced = 0
        self._t = threading.Thread(target=self._run, args=(iter(source),), daemon=True)
        self._t.start()

    @classmethod
    def from_iterator(cls, it, capacity: int = 4) -> "PrefetchIter":
        return cls(it, capacity)

    @classmethod
    def from_batches_bounded(cls, batches, capacity: int) -> "PrefetchIter":
        return cls(batches, capacity)

    def _put(self, item) -> bool:
        while not self._stop.is_set():
            try:
                self._q.put(item, timeout=0.05)
                return True
            except queue.Full:
                continue
        return False

    def _run(self, it):
        try:
            for x in it:
                if not self._put(x):
                    return
                self.produced += 1
            self._put(self._END)
        except BaseException as e:  # handed to the consumer
            self._put(("__error__", e))

    def __iter__(self):
        return self

    def __next__(self):
        x = self._q.get()
        if x is self._END:
            raise StopIteration
        if isinstance(x, tuple) and len(x) == 2 and x[0] == "__error__":
            raise x[1]
        return x

    def close(self) -> None:
        self._stop.set()


@dataclass
class StageProfile:
    name: str
    calls: int = 0
    total_s: float = 0.0

    @property
    def mean_ms(self) -> float:
        return 1e3 * self.total_s / self.calls if self.calls else 0.0


class MapStage:
    def __init__(self, name: str, fn):
        self.name, self.fn, self.profile = name, fn, StageProfile(name)

    def __call__(self, batch):
        t0 = time.perf_counter()
        out = self.fn(batch)
        self.profile.calls += 1
        self.profile.total_s += time.perf_counter() - t0
        return out


class PipelineRunner:
    """source -> stage 1 -> ... -> consumer, optionally prefetched; ``run_epoch`` returns the batch count."""

    def __init__(self, source_fn, prefetch: int = 0):
        self.source_fn, self.prefetch, self.stages = source_fn, prefetch, []

    def add_stage(self, name: str, fn) -> "PipelineRunner":
        self.stages.append(MapStage(name, fn))
        return self

    def process_batch(self, batch):
        for s in self.stages:
            batch = s(batch)
        return batch

    def iterate(self):
        gen = (self.process_batch(b) for b in self.source_fn())
        return PrefetchIter(gen, self.prefetch) if self.prefetch else gen

    def run_epoch(self, consume=None) -> int:
        n = 0
        for b in self.iterate():
            if consume:
                consume(b)
            n += 1
        return n

    def profiles(self) -> list[StageProfile]:
        return [s.profile for s in self.stages]


class MemoryLoader:
    """Batches of in-memory tensors (all indexed along dim 0), optionally shuffled per epoch."""

    def __init__(self, tensors, batch_size: int, shuffle: bool = False, seed: int = 0, drop_last: bool = False):
        self.tensors = list(tensors)
        n = self.tensors[0].shape[0]
        if any(t.shape[0] != n for t in self.tensors):
            raise ValueError("all tensors need the same leading size")
        self.n, self.bs, self.shuffle, self.seed, self.drop_last, self.epoch = n, batch_size, shuffle, seed, drop_last, 0

    @classmethod
    def from_tensors(cls, *tensors, batch_size: int = 32, **kw) -> "MemoryLoader":
        return cls(tensors, batch_size, **kw)

    def __len__(self):
        return self.n // self.bs if self.drop_last else -(-self.n // self.bs)

    def __iter__(self):
        idx = torch.tensor(shuffle_indices(self.n, self.seed + self.epoch)) if self.shuffle else torch.arange(self.n)
        self.epoch += 1
        for b in range(len(self)):
            sel = idx[b * self.bs:(b + 1) * self.bs]
            yield tuple(t[sel] for t in self.tensors)


class RandomImageDataset(Dataset):
    """Deterministic random images [C, H, W] in [0, 1) with integer labels (sample i seeded by seed + i)."""

    def __init__(self, n: int, channels: int = 3, size: int = 32, num_classes: int = 10, seed: int = 0):
        self.n, self.c, self.s, self.k, self.seed = n, channels, size, num_classes, seed

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        g = torch.Generator().manual_seed(self.seed + i)
        return torch.rand(self.c, self.s, self.s, generator=g), int(torch.randint(0, self.k, (), generator=g))


class RandomSegDataset(RandomImageDataset):
    """Images with dense label maps [H, W] (random axis-aligned class rectangles on background 0)."""

    def __getitem__(self, i):
        g = torch.Generator().manual_seed(self.seed + i)
        img = torch.rand(self.c, self.s, self.s, generator=g)
        mask = torch.zeros(self.s, self.s, dtype=torch.long)
        for _ in range(3):
            y0, x0 = torch.randint(0, self.s - 1, (2,), generator=g).tolist()
            h, w = torch.randint(1, self.s // 2 + 1, (2,), generator=g).tolist()
            mask[y0:y0 + h, x0:x0 + w] = int(torch.randint(1, self.k, (), generator=g))
        return img, mask


class SyntheticAudioDataset(Dataset):
    """Sine tones (class k = frequency base_hz * (k + 1)) with Gaussian noise, [samples] float32."""

    def __init__(self, n: int, sample_rate: int = 16000, seconds: float = 0.25, num_classes: int = 4,
                 base_hz: float = 220.0, noise: float = 0.05, seed: int = 0):
        self.n, self.sr, self.len, self.k, self.f0, self.noise, self.seed = (n, sample_rate, int(sample_rate * seconds),
                                                                             num_classes, base_hz, noise, seed)

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        g = torch.Generator().manual_seed(self.seed + i)
        k = int(torch.randint(0, self.k, (), generator=g))
        t = torch.arange(self.len) / self.sr
        x = torch.sin(2 * torch.pi * self.f0 * (k + 1) * t) + self.noise * torch.randn(self.len, generator=g)
        return x.float(), k
