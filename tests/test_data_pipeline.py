"""Prefetching, staged pipelines, in-memory loaders and synthetic datasets."""
import time

import pytest
import torch

from brain_b200.data import pipeline as P


def test_helpers():
    assert P.fnv_hash_bytes(b"") == 0xCBF29CE484222325 and P.fnv_hash_bytes(b"a") == 0xAF63DC4C8601EC8C
    assert P.dedup_items([3, 1, 3, 2, 1]) == [3, 1, 2]
    assert P.dedup_items(["a", "A", "b"], key=str.lower) == ["a", "b"]
    s = P.shuffle_indices(10, 7)
    assert sorted(s) == list(range(10)) and s == P.shuffle_indices(10, 7) and s != P.shuffle_indices(10, 8)
    x, lens = P.pad_and_stack_sequences([torch.tensor([1, 2, 3]), torch.tensor([4])], pad_value=-1)
    assert x.tolist() == [[1, 2, 3], [4, -1, -1]] and lens.tolist() == [3, 1]
    assert P.stack_samples_to_tensor([[1, 2], [3, 4]]).shape == (2, 2)
    calls = []
    lz = P.LazySample(lambda: calls.append(1) or 42)
    assert not lz.is_loaded and lz.get() == 42 and lz.get() == 42 and calls == [1]


def test_prefetch_backpressure_and_errors():
    produced = []

    def src():
        for i in range(10):
            produced.append(i)
            yield i
    it = P.PrefetchIter.from_batches_bounded(src(), capacity=2)
    time.sleep(0.2)
    assert len(produced) <= 4  # queue of 2 + one in the producer's hand + one being generated
    assert list(it) == list(range(10))

    def bad():
        yield 1
        raise RuntimeError("boom")
    it = P.PrefetchIter.from_iterator(bad())
    assert next(it) == 1
    with pytest.raises(RuntimeError, match="boom"):
        next(it)


def test_pipeline_runner_and_memory_loader():
    x = torch.arange(10.0)
    y = torch.arange(10) % 2
    ld = P.MemoryLoader.from_tensors(x, y, batch_size=4, shuffle=True, seed=3)
    b1 = [b[0].tolist() for b in ld]
    b2 = [b[0].tolist() for b in ld]
    assert len(ld) == 3 and sorted(sum(b1, [])) == list(range(10)) and b1 != b2
    with pytest.raises(ValueError):
        P.MemoryLoader([torch.ones(3), torch.ones(4)], 2)
    runner = P.PipelineRunner(lambda: iter(P.MemoryLoader.from_tensors(x, batch_size=3)), prefetch=2)
    runner.add_stage("double", lambda b: (b[0] * 2,)).add_stage("sum", lambda b: float(b[0].sum()))
    out = []
    assert runner.run_epoch(out.append) == 4 and sum(out) == 90.0
    assert [p.calls for p in runner.profiles()] == [4, 4] and runner.profiles()[0].mean_ms >= 0


def test_synthetic_datasets():
    ds = P.RandomImageDataset(5, channels=3, size=8, num_classes=4, seed=1)
    a, la = ds[2]
    b, lb = ds[2]
    assert a.shape == (3, 8, 8) and torch.equal(a, b) and la == lb and 0 <= la < 4
    img, mask = P.RandomSegDataset(3, size=16, num_classes=5)[0]
    assert mask.shape == (16, 16) and mask.max() < 5 and (mask > 0).any()
    au = P.SyntheticAudioDataset(4, sample_rate=8000, seconds=0.5, num_classes=3)
    w, k = au[1]
    spec = torch.fft.rfft(w).abs()
    peak_hz = int(spec.argmax()) * 8000 / w.numel()
    assert abs(peak_hz - 220 * (k + 1)) <= 4
    assert len(P.ConcatSources(ds, ds)) == 10
