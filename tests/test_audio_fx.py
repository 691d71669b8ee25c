"""Audio effects, augmentation, wavelets, codecs and frame features: the batched implementations against
per-sample loops that restate the reference's semantics (crates/brain-audio/src/augment/*.rs,
feature/wavelet.rs, encoding.rs, features_*.rs, vad.rs), plus the reference's own test vectors."""
import math

import numpy as np
import pytest
import torch

from brain_b200.zoo import audio_fx as A

SR = 8000


def _sig(n=2000, seed=0, batch=()):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*batch, n, generator=g, dtype=torch.float64) * 0.3


def _rround(v):
    return math.floor(v + 0.5)


def test_reverb_echo_chorus_vibrato_flanger_match_sample_loops():
    x = _sig(1500)
    xs = x.tolist()
    # Schroeder reverb: four combs, output = delay-line read
    out = [0.0] * len(xs)
    for ms in (0.0297, 0.0371, 0.0411, 0.0437):
        d = max(_rround(ms * SR), 1)
        g = 10.0 ** (-3.0 * (d / SR) / max(0.7, 0.1))
        buf, bi = [0.0] * d, 0
        for i, s in enumerate(xs):
            dl = buf[bi]
            buf[bi] = s + g * dl
            bi = (bi + 1) % d
            out[i] += 0.25 * dl
    torch.testing.assert_close(A.schroeder_reverb(x, SR, 0.7), torch.tensor(out, dtype=torch.float64))
    # multi-echo
    ref = list(xs)
    for d, gn in ((10, 0.5), (300, 0.25), (5000, 1.0)):
        if d < len(xs):
            for i in range(d, len(xs)):
                ref[i] += xs[i - d] * gn
    torch.testing.assert_close(A.multi_echo(x, [10, 300, 5000], [0.5, 0.25, 1.0]), torch.tensor(ref, dtype=torch.float64))
    # chorus
    base = _rround(15 * 1e-3 * SR)
    ref = list(xs)
    for i in range(len(xs)):
        cd = base * (1.0 + 0.5 * math.sin(2 * math.pi * 1.5 * i / SR))
        di = int(cd)
        if i > di:
            ref[i] += 0.5 * xs[i - di]
    torch.testing.assert_close(A.chorus(x, SR, 15, 1.5), torch.tensor(ref, dtype=torch.float64))
    # vibrato
    m = _rround(5 * 1e-3 * SR)
    ref = []
    for i in range(len(xs)):
        d = int(0.5 * (1 + math.sin(2 * math.pi * 4.0 * i / SR)) * m)
        ref.append(xs[i - d] if i >= d else 0.0)
    torch.testing.assert_close(A.vibrato(x, SR, 5, 4.0), torch.tensor(ref, dtype=torch.float64))
    # flanger: rotating buffer with feedback
    for depth in (3.0, 0.1):
        md = _rround(depth * 1e-3 * SR)
        buf = [0.0] * max(md, 1)
        ref = []
        for i in range(len(xs)):
            lfo = math.sin(2 * math.pi * 0.8 * i / SR)
            k = min(_rround(0.5 * (1 + lfo) * md), max(md - 1, 0))
            dl = buf[k]
            ref.append(xs[i] + dl)
            buf[0] = xs[i] + 0.6 * dl
            buf = [buf[-1]] + buf[:-1]
        torch.testing.assert_close(A.flanger(x, SR, depth, 0.8, 0.6), torch.tensor(ref, dtype=torch.float64))
    # batched input: every row filtered independently
    xb = _sig(600, 3, (3,))
    torch.testing.assert_close(A.flanger(xb, SR, 3.0, 0.8, 0.6)[1], A.flanger(xb[1], SR, 3.0, 0.8, 0.6))
    torch.testing.assert_close(A.schroeder_reverb(xb, SR, 0.5)[2], A.schroeder_reverb(xb[2], SR, 0.5))


@pytest.mark.parametrize("kind", ["low_pass", "high_pass", "band_pass", "notch"])
def test_biquad_matches_direct_form_one(kind):
    x = _sig(800, 4)
    b, a = A.biquad_coefficients(kind, SR, 900.0, 0.707)
    x1 = x2 = y1 = y2 = 0.0
    ref = []
    for x0 in x.tolist():
        y0 = (b[0] / a[0]) * x0 + (b[1] / a[0]) * x1 + (b[2] / a[0]) * x2 - (a[1] / a[0]) * y1 - (a[2] / a[0]) * y2
        ref.append(y0)
        x2, x1, y2, y1 = x1, x0, y1, y0
    torch.testing.assert_close(A.biquad_filter(x, kind, SR, 900.0, 0.707), torch.tensor(ref, dtype=torch.float64))


def test_time_domain_augmentations():
    x = _sig(1001, 5)
    y = A.time_stretch(x, 1.3)
    assert y.shape[-1] == _rround(1001 / 1.3)
    i = 17
    pos = min(i * 1.3, 1000.0)
    lo = math.floor(pos)
    torch.testing.assert_close(y[i], (1 - (pos - lo)) * x[lo] + (pos - lo) * x[min(lo + 1, 1000)])
    with pytest.raises(ValueError):
        A.time_stretch(x, 0.0)
    assert A.pitch_shift(x, 3.0).shape == x.shape
    z = A.time_mask(x.clone(), 990, 50)
    assert float(z[990:].abs().sum()) == 0.0 and torch.equal(z[:990], x[:990])
    # noise at the requested SNR, the reference's LCG + Box-Muller stream
    s = torch.sin(torch.arange(4000, dtype=torch.float64) * 0.05)
    noisy = A.add_noise(s.clone(), 10.0, 42)
    snr = 10 * math.log10(float(s.square().mean()) / float((noisy - s).square().mean()))
    assert abs(snr - 10.0) < 0.5
    state = (42 + 0x9E3779B97F4A7C15) & ((1 << 64) - 1)
    first = []
    for _ in range(3):
        vals = []
        for _ in range(2):
            state = (state * A._LCG_A + A._LCG_C) & ((1 << 64) - 1)
            vals.append(((state >> 32) + 1.0) / 4294967297.0)
        first.append(math.sqrt(-2 * math.log(vals[0])) * math.cos(2 * math.pi * vals[1]))
    std = math.sqrt(float(s.square().mean()) / 10.0)
    torch.testing.assert_close(noisy[:3] - s[:3], torch.tensor(first, dtype=torch.float64) * std)
    f = A.fade_out(A.fade_in(torch.ones(10, dtype=torch.float64), 4), 5)
    assert f.tolist() == pytest.approx([0.0, 0.25, 0.5, 0.75, 1.0, 1.0, 0.8, 0.6, 0.4, 0.2])
    assert A.clip_distortion(torch.tensor([-2.0, 0.1, 3.0]), -1.0).tolist() == pytest.approx([-1.0, 0.1, 1.0])
    assert A.gain_scale(torch.tensor([1.0, -2.0]), 0.5).tolist() == [0.5, -1.0]


def test_spectrogram_augmentations_follow_reference_draws():
    spec = torch.ones(40, 100, dtype=torch.float64)
    out = A.spec_augment_lcg(spec.clone(), 10, 2, 20, 2, seed=7)
    state, M = (7 + 0xDEADBEEF) & ((1 << 64) - 1), (1 << 64) - 1
    ref = spec.clone()

    def draw():
        nonlocal state
        state = (state * A._LCG_A + A._LCG_C) & M
        return state >> 32

    for size, param, axis in ((40, 10, 0), (100, 20, 1)):
        for _ in range(2):
            ln = draw() % min(param, size)
            st = draw() % max(size - ln, 1)
            if axis == 0:
                ref[st:st + ln] = 0
            else:
                ref[:, st:st + ln] = 0
    assert torch.equal(out, ref)
    c = A.spec_cutout(torch.ones(4, 6), 1, 2, 3, 10)
    assert float(c.sum()) == 24 - 6
    torch.testing.assert_close(A.spec_mixup(torch.ones(2, 2), torch.zeros(2, 2), 1.5), torch.ones(2, 2))
    with pytest.raises(ValueError):
        A.spec_mixup(torch.ones(2, 2), torch.ones(3, 2), 0.5)


def test_daubechies_filters_and_periodic_dwt():
    # the construction reproduces the published coefficients
    ref_db2 = [0.4829629131445341, 0.8365163037378079, 0.2241438680420134, -0.1294095225512604]
    assert np.allclose(A.daubechies_filter(4), ref_db2, atol=1e-14)
    ref_db4_head = [0.2303778133088965, 0.7148465705529157, 0.6308807679298589]
    assert np.allclose(A.daubechies_filter(8)[:3], ref_db4_head, atol=1e-13)
    for w in (A.WaveletType.HAAR, A.WaveletType.DB2, A.WaveletType.DB4, A.WaveletType.DB6, A.WaveletType.DB8):
        g = A.WaveletType.low_pass_filter(w)
        assert abs(float(g.sum()) - math.sqrt(2)) < 1e-12 and abs(float(g.square().sum()) - 1.0) < 1e-9
        x = _sig(64, w)
        a, d = A.dwt(x, w)
        h = A.WaveletType.high_pass_filter(w).tolist()
        gl = g.tolist()
        m = (64 + len(gl) - 1) // 2
        ra = [sum(float(x[(2 * i + k) % 64]) * gl[k] for k in range(len(gl))) for i in range(m)]
        rd = [sum(float(x[(2 * i + k) % 64]) * h[k] for k in range(len(gl))) for i in range(m)]
        torch.testing.assert_close(a, torch.tensor(ra, dtype=torch.float64))
        torch.testing.assert_close(d, torch.tensor(rd, dtype=torch.float64))
        if w == A.WaveletType.HAAR:  # orthogonal and no wrap-around: perfect reconstruction
            torch.testing.assert_close(A.idwt(a, d, w), x)
    torch.testing.assert_close(A.WaveletDenoise.soft_threshold(torch.tensor([-2.0, 0.3, 1.5]), 0.5),
                               torch.tensor([-1.5, 0.0, 1.0], dtype=torch.float64))


def test_companding_codecs_roundtrip_and_bit_layout():
    x = torch.linspace(-1, 1, 201, dtype=torch.float64)
    for enc, dec in ((A.mu_law_encode, A.mu_law_decode), (A.a_law_encode, A.a_law_decode)):
        c = enc(x)
        assert c.dtype == torch.uint8
        y = dec(c)
        assert float((y - x).abs().max()) < 0.03
        big = x.abs() > 0.05  # values that quantise to magnitude 0 decode as a signed zero
        assert bool((torch.sign(y[big]) == torch.sign(x[big])).all())
    # mu-law of +1.0: sign bit set, magnitude 127, then inverted -> 0x00; -1.0 -> 0x80
    assert A.mu_law_encode(torch.tensor([1.0, -1.0])).tolist() == [0x00, 0x80]
    assert A.a_law_encode(torch.tensor([1.0, -1.0])).tolist() == [0xFF ^ 0x55, 0x7F ^ 0x55]
    oh = A.phonetic_one_hot([2, 0, 2], 4)
    assert oh.shape == (4, 3) and oh[2, 0] == 1 and oh[0, 1] == 1 and float(oh.sum()) == 3
    with pytest.raises(IndexError):
        A.phonetic_one_hot([4], 4)


def test_frame_features_tempo_pitch_vad():
    x = _sig(1000, 9)
    r = A.rms_frames(x, 200, 100)
    assert r.shape == (9,)
    torch.testing.assert_close(r[3], x[300:500].square().mean().sqrt())
    assert A.rms_frames(x[:10], 200, 100).numel() == 0
    env = A.envelope_follower(x, SR, 5.0, 50.0)
    ga, gr = math.exp(-1 / max(5e-3 * SR, 1)), math.exp(-1 / max(50e-3 * SR, 1))
    cur, ref = 0.0, []
    for v in x.tolist():
        t = abs(v)
        cur = ga * cur + (1 - ga) * t if t > cur else gr * cur + (1 - gr) * t
        ref.append(cur)
    torch.testing.assert_close(env, torch.tensor(ref, dtype=torch.float64))
    # tempo: impulses every 25 frames at 50 frames/s -> 120 BPM
    onset = torch.zeros(400, dtype=torch.float64)
    onset[::25] = 1.0
    assert abs(A.estimate_tempo(onset, 50.0, 60.0, 200.0) - 120.0) < 1e-9
    assert A.estimate_tempo(onset[:10], 50.0) == 120.0
    # pitch: a 220 Hz tone
    t = torch.arange(1024, dtype=torch.float64) / SR
    f0 = A.pitch_autocorr(torch.sin(2 * math.pi * 220.0 * t), SR, 150.0, 500.0)  # 2 periods out of range
    assert f0 is not None and abs(f0 - 220.0) < 3.0
    assert A.pitch_autocorr(torch.zeros(30), SR, 80.0, 500.0) is None
    # VAD: silence, speech burst, silence; hysteresis holds speech through a short gap
    sig = torch.zeros(16000, dtype=torch.float64)
    sig[4000:9000] = torch.sin(torch.arange(5000, dtype=torch.float64) * 0.3)
    sig[6000:6300] = 0.0
    cfg = A.VADConfig()
    flags = A.compute_vad(sig, cfg)
    nf = (16000 - 512) // 160 + 1
    assert flags.shape == (nf,)
    assert not bool(flags[:20].any()) and bool(flags[30:50].all()) and not bool(flags[-10:].any())
    both = A.compute_vad(torch.stack([sig, torch.zeros_like(sig)]), cfg)
    assert torch.equal(both[0], flags) and not bool(both[1].any())
    trimmed = A.trim_silence(sig, -40.0, 512, 160)
    assert 4000 < trimmed.numel() < 16000 and float(trimmed[:100].abs().sum()) == 0.0
    # all silent: the start search runs off the end and the reference keeps the tail after the last frame start
    assert A.trim_silence(torch.zeros(3000), -40.0).numel() == 3000 - ((3000 - 512) // 160 + 1) * 160
