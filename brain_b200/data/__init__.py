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


# ------------------------------------------------------------------ native token loader
_LOADER_SIGS = {
    "brain_loader_open": ("brain_runtime", "piillliiiillp"),
    "brain_loader_next": ("brain_runtime", "ppp"),
    "brain_loader_fill": ("brain_runtime", "plp"),
    "brain_loader_stats": ("brain_runtime", "pp"),
    "brain_loader_close": ("brain_runtime", "p"),
}
_LOADER_ERRORS = {-10: "bad argument", -11: "I/O error", -12: "timed out waiting for a batch", -13: "closed"}


def _loader_fn(name):
    from .. import _native

    return _native.fn(name)


def _register_loader():
    from .. import _native

    _native.register(_LOADER_SIGS)


_register_loader()


def splitmix64_window_starts(seed: int, batch_index: int, rank: int, world: int, batch: int, seq: int,
                             n_tokens: int) -> list[int]:
    """Window starts of one batch, as the native loader draws them (the test oracle)."""
    m = (1 << 64) - 1
    st = (seed * 0x9E3779B97F4A7C15 + batch_index * world + rank) & m
    out = []
    for _ in range(batch):
        st = (st + 0x9E3779B97F4A7C15) & m
        z = st
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
        z ^= z >> 31
        out.append(z % (n_tokens - seq))
    return out


class NativeTokenLoader:
    """Random [batch, seq + 1] windows of a memory-mapped token file, assembled by C++ worker threads
    into a bounded ring (``depth`` batches ahead: back-pressure), copied into a pinned buffer per call.
    Iterating yields (inputs, targets) int64 CPU tensors; ``device=`` moves them with a non-blocking
    copy. Rank r of ``world`` draws its own stream; ``start_batch`` resumes a run at that batch."""

    def __init__(self, path: str, batch: int, seq: int, seed: int = 0, token_dtype=np.uint16, rank: int = 0,
                 world: int = 1, workers: int = 2, depth: int = 4, start_batch: int = 0, timeout_s: float = 60.0,
                 pin_memory: bool | None = None, device=None):
        import ctypes

        tb = np.dtype(token_dtype).itemsize
        h = ctypes.c_void_p()
        rc = _loader_fn("brain_loader_open")(path.encode(), tb, 8, batch, seq, seed, rank, world, workers, depth,
                                              start_batch, int(timeout_s * 1000), ctypes.byref(h))
        if rc != 0:
            raise RuntimeError(f"brain_loader_open({path}) failed: {_LOADER_ERRORS.get(rc, rc)}")
        self._h, self.batch, self.seq, self.device = h, batch, seq, device
        pin = torch.cuda.is_available() if pin_memory is None else pin_memory
        self._buf = torch.empty((batch, seq + 1), dtype=torch.int64, pin_memory=pin)
        self.last_batch_index = start_batch - 1

    def next(self):
        import ctypes

        if self._h is None:
            raise RuntimeError("loader is closed")
        idx = ctypes.c_int64(-1)
        rc = _loader_fn("brain_loader_next")(self._h, self._buf.data_ptr(), ctypes.byref(idx))
        if rc != 0:
            raise RuntimeError(f"brain_loader_next failed: {_LOADER_ERRORS.get(rc, rc)}")
        self.last_batch_index = idx.value
        w = self._buf
        if self.device is not None:
            w = w.to(self.device, non_blocking=True)
        else:
            w = w.clone()
        return w[:, :-1], w[:, 1:]

    def batch_at(self, b: int) -> torch.Tensor:
        out = torch.empty((self.batch, self.seq + 1), dtype=torch.int64)
        _loader_fn("brain_loader_fill")(self._h, b, out.data_ptr())
        return out

    def stats(self) -> dict:
        arr = (__import__("ctypes").c_int64 * 5)()
        _loader_fn("brain_loader_stats")(self._h, arr)
        return {"produced": arr[0], "consumed": arr[1], "consumer_wait_s": arr[2] * 1e-9,
                "producer_wait_s": arr[3] * 1e-9, "tokens": arr[4]}

    def checkpoint(self) -> "PipelineCheckpoint":
        return PipelineCheckpoint(0, self.last_batch_index + 1)

    def __iter__(self):
        while True:
            yield self.next()

    def close(self) -> None:
        if self._h is not None:
            _loader_fn("brain_loader_close")(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ samples, streams, caching, metrics
class Sample:
    """One record: data tensor, optional label and string metadata (brain-data core.rs:10-40)."""

    def __init__(self, id: int, data, label=None, meta=None):
        self.id, self.data, self.label, self.meta = id, data, label, dict(meta or {})

    def with_label(self, label) -> "Sample":
        self.label = label
        return self

    def with_meta(self, k, v) -> "Sample":
        self.meta[k] = v
        return self


def pad_collate(samples, pad_value: float = 0.0):
    """Pads variable-length [L, ...] sample tensors to the longest along dim 0 and stacks them;
    returns (batch, lengths[, labels])."""
    datas = [s.data if isinstance(s, Sample) else s for s in samples]
    L = max(d.shape[0] for d in datas)
    out = datas[0].new_full((len(datas), L) + tuple(datas[0].shape[1:]), pad_value)
    for i, d in enumerate(datas):
        out[i, :d.shape[0]] = d
    lengths = torch.tensor([d.shape[0] for d in datas])
    if samples and isinstance(samples[0], Sample) and samples[0].label is not None:
        return out, lengths, default_collate([s.label for s in samples])
    return out, lengths


class StreamDataset:
    """Iterable dataset over a generator factory; ``shard(rank, world)`` keeps every world-th record."""

    def __init__(self, make_iter, rank: int = 0, world: int = 1):
        self.make_iter, self.rank, self.world = make_iter, rank, world

    def shard(self, rank: int, world: int) -> "StreamDataset":
        return StreamDataset(self.make_iter, rank, world)

    def __iter__(self):
        for i, x in enumerate(self.make_iter()):
            if i % self.world == self.rank:
                yield x

    def batches(self, batch_size: int, drop_last: bool = False, collate=default_collate):
        buf = []
        for x in self:
            buf.append(x)
            if len(buf) == batch_size:
                yield collate(buf)
                buf = []
        if buf and not drop_last:
            yield collate(buf)


class ConcatDataset(Dataset):
    def __init__(self, *datasets):
        self.ds = datasets
        self.cum = np.cumsum([len(d) for d in datasets]).tolist()

    def __len__(self):
        return self.cum[-1] if self.cum else 0

    def __getitem__(self, i):
        k = int(np.searchsorted(self.cum, i, side="right"))
        return self.ds[k][i - (self.cum[k - 1] if k else 0)]


class SampleCache:
    """LRU cache of samples by index with hit / miss counters (brain-data caching.rs:10-40)."""

    def __init__(self, capacity: int):
        import collections

        self.capacity, self._d = capacity, collections.OrderedDict()
        self.hits = self.misses = 0

    def get(self, i):
        if i in self._d:
            self._d.move_to_end(i)
            self.hits += 1
            return self._d[i]
        self.misses += 1
        return None

    def put(self, i, v) -> None:
        self._d[i] = v
        self._d.move_to_end(i)
        while len(self._d) > self.capacity:
            self._d.popitem(last=False)


class CachedDataset(Dataset):
    def __init__(self, ds, capacity: int = 1024):
        self.ds, self.cache = ds, SampleCache(capacity)

    def __len__(self):
        return len(self.ds)

    def __getitem__(self, i):
        v = self.cache.get(i)
        if v is None:
            v = self.ds[i]
            self.cache.put(i, v)
        return v


class PipelineMetrics:
    """Samples / batches / seconds of a data pipeline and the consumer's time spent waiting on it."""

    def __init__(self):
        self.samples = self.batches = 0
        self.wait_s = 0.0
        self.t0 = None

    def wrap(self, it):
        import time

        self.t0 = time.perf_counter()
        it = iter(it)
        while True:
            t = time.perf_counter()
            try:
                b = next(it)
            except StopIteration:
                return
            self.wait_s += time.perf_counter() - t
            self.batches += 1
            first = b[0] if isinstance(b, (tuple, list)) else b
            self.samples += int(first.shape[0]) if hasattr(first, "shape") and first.dim() else 1
            yield b

    def throughput(self) -> float:
        import time

        el = time.perf_counter() - self.t0 if self.t0 else 0.0
        return self.samples / el if el > 0 else 0.0


class PipelineCheckpoint:
    """Position of a data pipeline (epoch, next sample / batch offset) for resuming."""

    def __init__(self, epoch: int = 0, sample_offset: int = 0):
        self.epoch, self.sample_offset = epoch, sample_offset

    def to_dict(self) -> dict:
        return {"epoch": self.epoch, "sample_offset": self.sample_offset}

    @classmethod
    def from_dict(cls, d) -> "PipelineCheckpoint":
        return cls(int(d["epoch"]), int(d["sample_offset"]))


def rle_encode(data) -> list[tuple[int, int]]:
    out = []
    for v in data:
        if out and out[-1][0] == v:
            out[-1] = (v, out[-1][1] + 1)
        else:
            out.append((v, 1))
    return out


def rle_decode(runs) -> list:
    return [v for v, n in runs for _ in range(n)]


def delta_encode(data) -> list[int]:
    return [data[0]] + [data[i] - data[i - 1] for i in range(1, len(data))] if len(data) else []


def delta_decode(d) -> list[int]:
    return np.cumsum(d).tolist() if len(d) else []
