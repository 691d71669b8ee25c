"""Dataset library: tabular (CSV), text-line, image-array and audio datasets, transforms, splits
(random / k-fold / stratified), class balancing, dataset statistics, a worker pool and a registry.

Reference: crates/brain-dataset (dataset/tabular.rs, text.rs, vision.rs, audio.rs; transforms/*.rs;
splits.rs:9-80; balance.rs:7-30; statistics.rs:7-30; loaders/worker.rs:6-30; the registry in
manage.rs). Records are torch tensors; batching and prefetch come from ``brain_b200.data.DataLoader``.
"""
from __future__ import annotations

import csv
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np
import torch

from . import Dataset


class TabularDataset(Dataset):
    """Numeric CSV; ``label_column`` (name or index, default last) is returned as an int64 label for
    classification or as a float target when ``regression``."""

    def __init__(self, path: str, label_column=-1, header: bool | None = None, regression: bool = False,
                 transform=None):
        with open(path, newline="") as f:
            rows = [r for r in csv.reader(f) if r and not r[0].startswith("#")]
        if header is None:
            try:
                [float(v) for v in rows[0]]
                header = False
            except ValueError:
                header = True
        self.columns = rows[0] if header else [f"c{i}" for i in range(len(rows[0]))]
        body = rows[1:] if header else rows
        li = self.columns.index(label_column) if isinstance(label_column, str) else label_column % len(self.columns)
        arr = np.array([[float(v) for v in r] for r in body], dtype=np.float32)
        self.x = torch.from_numpy(np.delete(arr, li, axis=1))
        y = torch.from_numpy(arr[:, li])
        self.y = y if regression else y.to(torch.int64)
        self.feature_names = [c for i, c in enumerate(self.columns) if i != li]
        self.transform = transform

    def __len__(self):
        return self.x.shape[0]

    def __getitem__(self, i):
        x = self.x[i]
        return (self.transform(x) if self.transform else x), self.y[i]


class TextLineDataset(Dataset):
    """One example per non-empty line; optional tokenizer (``brain_b200.text``) turns lines into ids,
    ``max_len`` truncates, and ``label_sep`` splits "label<sep>text" lines."""

    def __init__(self, path: str, tokenizer=None, max_len: int = 0, label_sep: str | None = None):
        with open(path, encoding="utf-8") as f:
            lines = [ln.rstrip("\n") for ln in f if ln.strip()]
        self.labels = None
        if label_sep is not None:
            parts = [ln.split(label_sep, 1) for ln in lines]
            names = sorted({p[0] for p in parts})
            self.label_names = names
            self.labels = [names.index(p[0]) for p in parts]
            lines = [p[1] if len(p) > 1 else "" for p in parts]
        self.lines, self.tok, self.max_len = lines, tokenizer, max_len

    def __len__(self):
        return len(self.lines)

    def __getitem__(self, i):
        x = self.lines[i]
        if self.tok is not None:
            ids = self.tok.encode(x).ids
            if self.max_len:
                ids = ids[:self.max_len]
            x = torch.tensor(ids, dtype=torch.int64)
        return (x, self.labels[i]) if self.labels is not None else x


class ImageArrayDataset(Dataset):
    """Images stored as ``.npy`` arrays [H, W, C] (uint8 or float) in ``root/<class>/`` folders; returns
    ([C, H, W] float in [0, 1] for uint8, transformed), class index."""

    def __init__(self, root: str, transform=None):
        self.classes = sorted(d for d in os.listdir(root) if os.path.isdir(os.path.join(root, d)))
        self.items = [(os.path.join(root, c, f), k) for k, c in enumerate(self.classes)
                      for f in sorted(os.listdir(os.path.join(root, c))) if f.endswith(".npy")]
        self.transform = transform

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        path, k = self.items[i]
        a = np.load(path)
        t = torch.from_numpy(a).permute(2, 0, 1)
        t = t.float() / 255.0 if a.dtype == np.uint8 else t.float()
        return (self.transform(t) if self.transform else t), k


class AudioDataset(Dataset):
    """16-bit PCM WAV files in ``root/<class>/``; returns (features, class index) with ``features`` from
    ``transform`` (e.g. ``zoo.audio.mfcc``) or the raw mono waveform."""

    def __init__(self, root: str, transform=None, sample_rate: int | None = None):
        self.classes = sorted(d for d in os.listdir(root) if os.path.isdir(os.path.join(root, d)))
        self.items = [(os.path.join(root, c, f), k) for k, c in enumerate(self.classes)
                      for f in sorted(os.listdir(os.path.join(root, c))) if f.endswith(".wav")]
        self.transform, self.sample_rate = transform, sample_rate

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        from ..zoo.audio import read_wav, resample

        path, k = self.items[i]
        x, sr = read_wav(path)
        x = x.mean(0)
        if self.sample_rate and sr != self.sample_rate:
            x = resample(x, sr, self.sample_rate)
        return (self.transform(x) if self.transform else x), k


# ------------------------------------------------------------------ transforms
class Compose:
    def __init__(self, *fns):
        self.fns = fns

    def __call__(self, x):
        for f in self.fns:
            x = f(x)
        return x


class Normalize:
    def __init__(self, mean, std):
        self.mean, self.std = torch.as_tensor(mean), torch.as_tensor(std)

    def __call__(self, x):
        shape = (-1,) + (1,) * (x.dim() - 1) if self.mean.dim() and x.dim() > 1 else ()
        m = self.mean.view(shape) if shape else self.mean
        s = self.std.view(shape) if shape else self.std
        return (x - m) / s


class MinMaxScale:
    def __init__(self, lo, hi):
        self.lo, self.hi = torch.as_tensor(lo), torch.as_tensor(hi)

    def __call__(self, x):
        return (x - self.lo) / (self.hi - self.lo).clamp_min(1e-12)


class RandomHorizontalFlip:
    def __init__(self, p: float = 0.5, seed: int = 0):
        self.p, self.g = p, torch.Generator().manual_seed(seed)

    def __call__(self, x):
        return x.flip(-1) if float(torch.rand(1, generator=self.g)) < self.p else x


class RandomCrop:
    def __init__(self, size: int, padding: int = 0, seed: int = 0):
        self.size, self.padding, self.g = size, padding, torch.Generator().manual_seed(seed)

    def __call__(self, x):
        if self.padding:
            x = torch.nn.functional.pad(x, (self.padding,) * 4)
        H, W = x.shape[-2:]
        y0 = int(torch.randint(0, H - self.size + 1, (1,), generator=self.g))
        x0 = int(torch.randint(0, W - self.size + 1, (1,), generator=self.g))
        return x[..., y0:y0 + self.size, x0:x0 + self.size]


class AddGaussianNoise:
    def __init__(self, std: float, seed: int = 0):
        self.std, self.g = std, torch.Generator().manual_seed(seed)

    def __call__(self, x):
        return x + torch.randn(x.shape, generator=self.g, dtype=x.dtype) * self.std


class Lowercase:
    def __call__(self, s: str) -> str:
        return s.lower()


# ------------------------------------------------------------------ splits / balance / statistics
@dataclass
class SplitResult:
    train: list
    val: list
    test: list


def random_split_indices(total: int, train_frac: float, val_frac: float, seed: int = 0) -> SplitResult:
    perm = torch.randperm(total, generator=torch.Generator().manual_seed(seed)).tolist()
    nt = int(total * train_frac)
    nv = int(total * val_frac)
    return SplitResult(perm[:nt], perm[nt:nt + nv], perm[nt + nv:])


def k_fold_split_indices(total: int, k: int):
    """k (train, val) pairs; fold i validates on the i-th contiguous chunk (sizes differ by at most 1)."""
    bounds = [round(i * total / k) for i in range(k + 1)]
    idx = list(range(total))
    return [(idx[:bounds[i]] + idx[bounds[i + 1]:], idx[bounds[i]:bounds[i + 1]]) for i in range(k)]


def stratified_split_indices(labels, train_frac: float, seed: int = 0):
    """Per class, the first round(n_c * train_frac) of a seeded shuffle go to train."""
    g = torch.Generator().manual_seed(seed)
    labels = list(labels)
    train, val = [], []
    for c in sorted(set(labels)):
        idx = [i for i, y in enumerate(labels) if y == c]
        idx = [idx[j] for j in torch.randperm(len(idx), generator=g).tolist()]
        k = int(round(len(idx) * train_frac))
        train += idx[:k]
        val += idx[k:]
    return sorted(train), sorted(val)


def balance_indices(labels, target_per_class: int | None = None, seed: int = 0):
    """Over- / under-samples every class to ``target_per_class`` (default: the largest class)."""
    g = torch.Generator().manual_seed(seed)
    labels = list(labels)
    by = {}
    for i, y in enumerate(labels):
        by.setdefault(y, []).append(i)
    t = target_per_class or max(len(v) for v in by.values())
    out = []
    for c in sorted(by):
        idx = by[c]
        if len(idx) >= t:
            out += [idx[j] for j in torch.randperm(len(idx), generator=g)[:t].tolist()]
        else:
            out += [idx[j] for j in torch.randint(0, len(idx), (t,), generator=g).tolist()]
    return out


@dataclass
class DatasetStats:
    total_samples: int
    num_classes: int
    class_counts: dict
    feature_mean: torch.Tensor | None = None
    feature_std: torch.Tensor | None = None

    def imbalance_ratio(self) -> float:
        c = [v for v in self.class_counts.values() if v]
        return max(c) / min(c) if c else 1.0


def dataset_stats(ds) -> DatasetStats:
    xs, counts = [], {}
    for i in range(len(ds)):
        x, y = ds[i]
        y = int(y)
        counts[y] = counts.get(y, 0) + 1
        if isinstance(x, torch.Tensor) and x.is_floating_point():
            xs.append(x.reshape(-1))
    mean = std = None
    if xs and all(x.shape == xs[0].shape for x in xs):
        st = torch.stack(xs)
        mean, std = st.mean(0), st.std(0, unbiased=False)
    return DatasetStats(len(ds), len(counts), counts, mean, std)


class WorkerPool:
    """Maps a function over items on ``num_workers`` threads, results in input order."""

    def __init__(self, num_workers: int = 4):
        self.num_workers = max(1, num_workers)

    def map(self, fn, items):
        with ThreadPoolExecutor(self.num_workers) as ex:
            return list(ex.map(fn, items))

    def load(self, ds, indices):
        return self.map(ds.__getitem__, indices)


# ------------------------------------------------------------------ registry
_REGISTRY: dict = {}


def register_dataset(name: str, factory) -> None:
    if name in _REGISTRY:
        raise KeyError(f"dataset '{name}' is already registered")
    _REGISTRY[name] = factory


def create_dataset(name: str, **kw):
    if name not in _REGISTRY:
        raise KeyError(f"unknown dataset '{name}'; registered: {sorted(_REGISTRY)}")
    return _REGISTRY[name](**kw)


def list_datasets() -> list[str]:
    return sorted(_REGISTRY)


def _register_builtin():
    from . import SyntheticImages, SyntheticTokens

    register_dataset("synthetic_tokens", lambda **kw: SyntheticTokens(**kw))
    register_dataset("synthetic_images", lambda **kw: SyntheticImages(**kw))
    register_dataset("csv", lambda path, **kw: TabularDataset(path, **kw))
    register_dataset("text_lines", lambda path, **kw: TextLineDataset(path, **kw))
    register_dataset("image_arrays", lambda root, **kw: ImageArrayDataset(root, **kw))
    register_dataset("audio", lambda root, **kw: AudioDataset(root, **kw))


_register_builtin()
