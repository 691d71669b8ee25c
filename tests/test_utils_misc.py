"""Process-level utilities (crates/brain-utils/src/utils.rs, io/, fs_stats.rs, serialize_helpers.rs,
hash.rs, config/schema.rs, version.rs, env.rs, metrics_utils.rs, prof/)."""
import os

import pytest

from brain_b200.utils import misc as U


def test_rate_limiter_and_retry():
    t = [0.0]
    rl = U.TokenBucketRateLimiter(rate=10.0, burst=2.0, clock=lambda: t[0])
    assert rl.try_acquire() and rl.try_acquire() and not rl.try_acquire()
    t[0] += 0.1
    assert rl.try_acquire() and not rl.try_acquire()
    slept = []

    def sleep(d):
        slept.append(d)
        t[0] += d

    rl.acquire(1.0, sleep=sleep)
    assert slept and sum(slept) >= 0.1 - 1e-9
    calls = []

    def flaky():
        calls.append(1)
        if len(calls) < 3:
            raise RuntimeError("x")
        return 7

    delays = []
    assert U.retry_with_backoff(flaky, attempts=5, base_delay=0.1, jitter=0.0, sleep=delays.append) == 7
    assert delays == pytest.approx([0.1, 0.2])
    with pytest.raises(RuntimeError):
        U.retry_with_backoff(lambda: (_ for _ in ()).throw(RuntimeError("y")), attempts=2, sleep=lambda d: None)


def test_files_and_dir_stats(tmp_path):
    p = str(tmp_path / "a" / "b.txt")
    U.ensure_dir(os.path.dirname(p))
    U.atomic_write_file(p, b"hello")
    U.append_file(p, " world")
    assert open(p).read() == "hello world"
    assert [f for f in os.listdir(os.path.dirname(p)) if f.startswith(".tmp-")] == []
    st = U.scan_dir_stats(str(tmp_path))
    assert st.files == 1 and st.bytes == 11 and st.by_extension == {".txt": 1} and st.largest_file == p
    assert U.dir_size(str(tmp_path)) == 11 and U.file_count(str(tmp_path)) == 1
    assert U.sanitize_filename("../a b?.txt") == "_a_b_.txt" and U.sanitize_filename("...") == "unnamed"
    assert U.normalize_slashes("a\\\\b//c") == "a/b/c"
    with pytest.raises(ValueError):
        U.join_safe(str(tmp_path), "..", "etc")
    assert U.join_safe(str(tmp_path), "a", "b.txt") == os.path.realpath(p)
    assert U.unique_temp_path("x", ".bin") != U.unique_temp_path("x", ".bin")


def test_formatting_parsing_encoding():
    assert U.parse_size("4k") == 4000 and U.parse_size("1.5 MB") == 1_500_000 and U.parse_size("2GiB") == 2 * 2 ** 30
    with pytest.raises(ValueError):
        U.parse_size("3 parsecs")
    assert U.format_bytes(1536, binary=True) == "1.50 KiB" and U.format_bytes(999) == "999 B"
    assert U.format_duration(0.00123) == "1.23 ms" and U.format_duration(3723) == "1h 02m 03s"
    assert U.parse_duration("1h30m") == 5400 and U.parse_duration("250ms") == pytest.approx(0.25)
    with pytest.raises(ValueError):
        U.parse_duration("soon")
    assert U.format_percent(0.1234) == "12.3%" and U.truncate_str("abcdef", 5) == "ab..."
    assert U.shell_quote("a b'c") == "'a b'\"'\"'c'" and U.shell_quote("ok.txt") == "ok.txt"
    assert U.base64_decode(U.base64_encode(b"\x00\xff")) == b"\x00\xff" and U.hex_to_bytes(U.bytes_to_hex(b"ab")) == b"ab"
    assert U.hash_combine_64(1, 2) != U.hash_combine_64(2, 1)
    assert len(U.random_uuid_lite()) == 36


def test_schema_version_system_metrics_timing():
    v = U.SchemaValidator([U.FieldDef("lr", "float", constraint=U.Constraint(min=0, max=1)),
                           U.FieldDef("opt", "str", constraint=U.Constraint(choices=("adam", "sgd"))),
                           U.FieldDef("steps", "int", required=False, default=10)], strict=True)
    cfg, errs = v.validate({"lr": 0.1, "opt": "adam"})
    assert errs == [] and cfg["steps"] == 10
    _, errs = v.validate({"lr": 2.0, "opt": "lion", "x": 1})
    assert len(errs) == 3
    _, errs = v.validate({"lr": True, "opt": "adam"})
    assert errs and "expected float" in errs[0]
    assert U.Version.parse("v1.2.3") < U.Version.parse("1.10") and str(U.Version.parse("2")) == "2.0.0"
    assert U.Version(1, 2).is_compatible(U.Version(1, 9)) and not U.Version(0, 1).is_compatible(U.Version(0, 2))
    si = U.SystemInfo.collect()
    assert si.cpu_count >= 1 and si.torch
    m = U.MetricsRegistry()
    m.inc("req")
    m.inc("req", 2)
    m.set("temp", 40.5)
    for x in range(101):
        m.observe("lat", x)
    snap = m.snapshot()
    assert snap["req"] == 3 and snap["temp"] == 40.5 and snap["lat"]["p50"] == 50 and snap["lat"]["p99"] == 99
    with pytest.raises(ValueError):
        m.set("req", 1)
    t = [0.0]
    tree = U.TimingTree(clock=lambda: t[0])
    with tree.section("step"):
        with tree.section("fwd"):
            t[0] += 0.5
        t[0] += 0.25
    rep = tree.report()
    assert "step: 1 call(s), 750.00 ms" in rep and "  fwd: 1 call(s), 500.00 ms" in rep


def test_nn_activation_and_init_extras():
    import math

    import torch

    from brain_b200.nn import init as I
    from brain_b200.nn import layers as L
    x = torch.tensor([-2.0, -0.3, 0.0, 0.4, 1.5])
    assert L.CELU(2.0)(x).tolist() == pytest.approx([2 * math.expm1(-1.0), 2 * math.expm1(-0.15), 0.0, 0.4, 1.5])
    assert L.HardShrink(0.5)(x).tolist() == [-2.0, 0.0, 0.0, 0.0, 1.5]
    assert L.SoftShrink(0.5)(x).tolist() == pytest.approx([-1.5, 0.0, 0.0, 0.0, 1.0])
    assert L.Shrink(0.5, 0.25)(x).tolist() == pytest.approx([-1.75, 0.0, 0.0, 0.0, 1.25])
    assert L.ThresholdedReLU(1.0)(x).tolist() == [0.0, 0.0, 0.0, 0.0, 1.5]
    assert L.TanhShrink()(x)[4].item() == pytest.approx(1.5 - math.tanh(1.5))
    assert torch.allclose(L.Softmin()(x), torch.softmax(-x, -1))
    q = L.QuietSoftmax()(x[None])
    s = x / (1 + torch.exp(x))
    assert torch.allclose(q[0], torch.softmax(s, -1)) and float(q.sum()) == pytest.approx(1.0)
    fd = L.FusedDropout(0.5).eval()
    assert torch.equal(fd(x, torch.ones(5)), x + 1)
    seq = L.SequentialNamed([("a", L.ThresholdedReLU(0.0)), ("b", L.TanhShrink())])
    assert hasattr(seq, "a") and torch.allclose(seq(x), L.TanhShrink()(L.ThresholdedReLU(0.0)(x)))
    assert I.calculate_fan((16, 8, 3, 3)) == (72, 144) and I.calculate_fan((5,)) == (5, 5)
    assert torch.allclose(I.scaled_residual_init(torch.ones(2), 8), torch.full((2,), 0.25))
    assert float(I.zero_init_last_layer((3, 4)).abs().sum()) == 0.0
