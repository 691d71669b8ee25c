"""Audio augmentation, effects, codecs, wavelets and frame-level features, batched over leading dims.

Reference: crates/brain-audio/src/augment/effects.rs (Schroeder reverb, multi-echo, chorus, flanger,
vibrato, biquad filters), augment/time.rs (time stretch, pitch shift, masks, noise at a target SNR,
gain, clipping, fades), augment/spectral.rs (SpecAugment masks, cutout, mixup), feature/wavelet.rs
(periodic DWT/IDWT with Haar and Daubechies filters, soft-threshold denoising), encoding.rs (mu-law and
A-law companding, phonetic one-hot), features_energy.rs (frame RMS, envelope follower),
features_rhythm.rs (autocorrelation tempo), features_pitch.rs (normalised-autocorrelation pitch with
parabolic refinement) and vad.rs (energy VAD with hysteresis, silence trimming).

Every function takes a tensor whose LAST dimension is time and works on all leading dimensions at
once: feed-forward effects are gathers and shifted adds over the whole batch, recursive filters run
``scipy.signal.lfilter`` along time for every row together, and the few recursions with a
time-varying delay or branch (flanger, envelope follower) step through time with one vector
operation per sample over the batch. The reference processes one ``&[f64]`` at a time. Results
match its per-signal outputs (float64).

The Daubechies filters are not a stored table: ``daubechies_filter(taps)`` builds them by the
published spectral-factorisation construction (Daubechies 1988): the roots of the half-band
polynomial inside the unit circle give the minimum-phase filter, normalised to sum sqrt(2).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from functools import lru_cache

import numpy as np
import torch

from ..utils.random import LCG64_A as _LCG_A, LCG64_C as _LCG_C, lcg64_stream

_M64 = (1 << 64) - 1


def _rnd(v: float) -> int:
    """Round half away from zero (Rust's f64::round; Python's round() goes to even), v >= 0."""
    return int(math.floor(v + 0.5))


def _f64(x) -> torch.Tensor:
    return torch.as_tensor(x, dtype=torch.float64)


def _shift(x: torch.Tensor, d: int) -> torch.Tensor:
    """x delayed by d samples along time, zeros shifted in."""
    if d <= 0:
        return x
    out = torch.zeros_like(x)
    if d < x.shape[-1]:
        out[..., d:] = x[..., :-d]
    return out


def _lfilter(b, a, x: torch.Tensor) -> torch.Tensor:
    from scipy.signal import lfilter
    y = lfilter(np.asarray(b, dtype=np.float64), np.asarray(a, dtype=np.float64), x.detach().cpu().double().numpy(),
                axis=-1)
    return torch.from_numpy(np.ascontiguousarray(y)).to(x.device)


# ------------------------------------------------------------------------------------------ effects
def schroeder_reverb(signal: torch.Tensor, sample_rate: int, decay_time_sec: float) -> torch.Tensor:
    """Mean of four feedback combs (29.7, 37.1, 41.1, 43.7 ms) whose gains give a 60 dB decay over
    decay_time_sec (at least 0.1 s); each comb's output is its delay line's read (y[n - D])."""
    x = _f64(signal)
    if x.shape[-1] == 0:
        return x.clone()
    sr = float(sample_rate)
    out = torch.zeros_like(x)
    for ms in (0.0297, 0.0371, 0.0411, 0.0437):
        d = max(_rnd(ms * sr), 1)
        g = 10.0 ** (-3.0 * (d / sr) / max(decay_time_sec, 0.1))
        a = np.zeros(d + 1)
        a[0], a[d] = 1.0, -g
        y = _lfilter([1.0], a, x)  # y[n] = x[n] + g y[n - d]
        out += 0.25 * _shift(y, d)
    return out


def multi_echo(signal: torch.Tensor, delays, gains) -> torch.Tensor:
    """x + sum_k gains[k] * x delayed by delays[k] (delays beyond the signal are ignored)."""
    x = _f64(signal)
    out = x.clone()
    for d, g in zip(delays, gains):
        if int(d) < x.shape[-1]:
            out += float(g) * _shift(x, int(d))
    return out


def _lfo(n: int, sample_rate: int, rate_hz: float, device=None) -> torch.Tensor:
    i = torch.arange(n, dtype=torch.float64, device=device)
    return torch.sin(2.0 * math.pi * rate_hz * i / float(sample_rate))


def _gather_delayed(x: torch.Tensor, delay: torch.Tensor, valid: torch.Tensor) -> torch.Tensor:
    idx = (torch.arange(x.shape[-1], device=x.device) - delay).clamp_min(0)
    g = x.index_select(-1, idx)
    return torch.where(valid, g, torch.zeros_like(g))


def chorus(signal: torch.Tensor, sample_rate: int, depth_ms: float, rate_hz: float) -> torch.Tensor:
    """x[i] + 0.5 x[i - d(i)] with d(i) = floor(D (1 + 0.5 sin(2 pi f i / sr))), D = depth in samples;
    added only where i > d(i)."""
    x = _f64(signal)
    n = x.shape[-1]
    base = _rnd(depth_ms * 1e-3 * sample_rate)
    d = (base * (1.0 + 0.5 * _lfo(n, sample_rate, rate_hz, x.device))).floor().long()
    i = torch.arange(n, device=x.device)
    return x + 0.5 * _gather_delayed(x, d, i > d)


def vibrato(signal: torch.Tensor, sample_rate: int, depth_ms: float, rate_hz: float) -> torch.Tensor:
    """x[i - d(i)] with d(i) = floor(0.5 (1 + sin(2 pi f i / sr)) M), M = depth in samples (0 before the start)."""
    x = _f64(signal)
    n = x.shape[-1]
    m = _rnd(depth_ms * 1e-3 * sample_rate)
    d = (0.5 * (1.0 + _lfo(n, sample_rate, rate_hz, x.device)) * m).floor().long()
    i = torch.arange(n, device=x.device)
    return _gather_delayed(x, d, i >= d)


def flanger(signal: torch.Tensor, sample_rate: int, depth_ms: float, rate_hz: float, feedback: float) -> torch.Tensor:
    """Feedback comb with a swept delay: w[t] = x[t] + feedback * r[t], out[t] = x[t] + r[t], where r[t]
    reads w at lag k(t) = min(round(0.5 (1 + sin) M), M - 1) (lag 0 reads the oldest slot, M back)."""
    x = _f64(signal)
    n = x.shape[-1]
    mraw = _rnd(depth_ms * 1e-3 * sample_rate)
    m = max(mraw, 1)
    k = torch.floor(0.5 * (1.0 + _lfo(n, sample_rate, rate_hz)) * mraw + 0.5).long().clamp(max=max(mraw - 1, 0)).tolist()
    xs = x.reshape(-1, n).cpu().numpy()
    w = np.zeros_like(xs)
    out = np.empty_like(xs)
    for t in range(n):
        lag = k[t] if k[t] >= 1 else m
        r = w[:, t - lag] if t - lag >= 0 else 0.0
        out[:, t] = xs[:, t] + r
        w[:, t] = xs[:, t] + feedback * r
    return torch.from_numpy(out).view_as(x).to(x.device)


class BiquadType:
    LOW_PASS, HIGH_PASS, BAND_PASS, NOTCH = "low_pass", "high_pass", "band_pass", "notch"


def biquad_coefficients(filter_type: str, sample_rate: int, cutoff_hz: float, q: float):
    """(b, a) of the RBJ audio-EQ-cookbook biquad (Q at least 0.1), not yet normalised by a0."""
    w0 = 2.0 * math.pi * cutoff_hz / sample_rate
    alpha = math.sin(w0) / (2.0 * max(q, 0.1))
    c = math.cos(w0)
    a = [1.0 + alpha, -2.0 * c, 1.0 - alpha]
    b = {BiquadType.LOW_PASS: [(1 - c) / 2, 1 - c, (1 - c) / 2],
         BiquadType.HIGH_PASS: [(1 + c) / 2, -(1 + c), (1 + c) / 2],
         BiquadType.BAND_PASS: [alpha, 0.0, -alpha],
         BiquadType.NOTCH: [1.0, -2.0 * c, 1.0]}[filter_type]
    return b, a


def biquad_filter(signal: torch.Tensor, filter_type: str, sample_rate: int, cutoff_hz: float, q: float) -> torch.Tensor:
    b, a = biquad_coefficients(filter_type, sample_rate, cutoff_hz, q)
    return _lfilter([v / a[0] for v in b], [1.0, a[1] / a[0], a[2] / a[0]], _f64(signal))


# ------------------------------------------------------------------------------------------ time domain
def time_stretch(signal: torch.Tensor, rate: float) -> torch.Tensor:
    """Resample to round(n / rate) samples by linear interpolation at positions i * rate (clamped)."""
    if rate <= 0.0:
        raise ValueError("time_stretch rate must be > 0.0")
    x = _f64(signal)
    n = x.shape[-1]
    if n == 0:
        return x.clone()
    m = _rnd(n / rate)
    if m == 0:
        return x[..., :1].clone()
    pos = (torch.arange(m, dtype=torch.float64, device=x.device) * rate).clamp(max=n - 1.0)
    lo = pos.floor().long()
    hi = (lo + 1).clamp(max=n - 1)
    frac = pos - lo.double()
    return (1.0 - frac) * x.index_select(-1, lo) + frac * x.index_select(-1, hi)


def pitch_shift(signal: torch.Tensor, semitones: float) -> torch.Tensor:
    """Stretch by 2^(-semitones/12), then stretch back to the original length (pitch moves, duration stays)."""
    x = _f64(signal)
    s = time_stretch(x, 2.0 ** (-semitones / 12.0))
    return time_stretch(s, s.shape[-1] / x.shape[-1])


def time_mask(signal: torch.Tensor, start: int, mask_len: int) -> torch.Tensor:
    """Zero samples [start, start + mask_len) in place (clipped to the signal); returns the signal."""
    n = signal.shape[-1]
    signal[..., min(start, n):min(start + mask_len, n)] = 0.0
    return signal


def add_noise(signal: torch.Tensor, snr_db: float, seed: int) -> torch.Tensor:
    """Add Gaussian noise at the given SNR (signal power / noise power) in place, per row, with the
    reference's generator: state = seed + 0x9e3779b97f4a7c15, then per sample two LCG draws
    u = ((state >> 32) + 1) / (2^32 + 1) and a Box-Muller cosine normal. Every row uses the same stream."""
    n = signal.shape[-1]
    if n == 0:
        return signal
    x = _f64(signal)
    power = x.square().mean(-1, keepdim=True)
    std = (power / max(10.0 ** (snr_db / 10.0), 1e-6)).sqrt()
    st = lcg64_stream((seed + 0x9E3779B97F4A7C15) & _M64, 2 * n)
    u = ((st >> np.uint64(32)).astype(np.float64) + 1.0) / 4294967297.0
    normal = np.sqrt(-2.0 * np.log(u[0::2])) * np.cos(2.0 * math.pi * u[1::2])
    signal.copy_((x + std * torch.from_numpy(normal).to(x.device)).to(signal.dtype))
    return signal


def gain_scale(signal: torch.Tensor, gain: float) -> torch.Tensor:
    return signal.mul_(gain)


def clip_distortion(signal: torch.Tensor, limit: float) -> torch.Tensor:
    lim = abs(limit)
    return signal.clamp_(-lim, lim)


def fade_in(signal: torch.Tensor, fade_len: int) -> torch.Tensor:
    """Scale the first L = min(fade_len, n) samples by i / L in place."""
    L = min(fade_len, signal.shape[-1])
    if L:
        signal[..., :L] *= torch.arange(L, dtype=torch.float64, device=signal.device).div(L).to(signal.dtype)
    return signal


def fade_out(signal: torch.Tensor, fade_len: int) -> torch.Tensor:
    """Scale the last L samples by 1 - i / L in place."""
    n = signal.shape[-1]
    L = min(fade_len, n)
    if L:
        signal[..., n - L:] *= (1.0 - torch.arange(L, dtype=torch.float64, device=signal.device) / L).to(signal.dtype)
    return signal


# ------------------------------------------------------------------------------------------ spectrogram
def frequency_mask(spec: torch.Tensor, f_start: int, f_len: int) -> torch.Tensor:
    """Zero bins [f_start, f_start + f_len) of a [.., freq, time] spectrogram in place."""
    spec[..., f_start:min(f_start + f_len, spec.shape[-2]), :] = 0.0
    return spec


def time_mask_spec(spec: torch.Tensor, t_start: int, t_len: int) -> torch.Tensor:
    spec[..., t_start:min(t_start + t_len, spec.shape[-1])] = 0.0
    return spec


def spec_cutout(spec: torch.Tensor, f_start: int, f_len: int, t_start: int, t_len: int) -> torch.Tensor:
    spec[..., f_start:min(f_start + f_len, spec.shape[-2]), t_start:min(t_start + t_len, spec.shape[-1])] = 0.0
    return spec


def spec_mixup(spec1: torch.Tensor, spec2: torch.Tensor, alpha: float) -> torch.Tensor:
    """a spec1 + (1 - a) spec2 with a = clamp(alpha, 0, 1)."""
    if spec1.shape != spec2.shape:
        raise ValueError(f"spec_mixup shapes differ: {tuple(spec1.shape)} vs {tuple(spec2.shape)}")
    a = min(max(alpha, 0.0), 1.0)
    return a * spec1 + (1.0 - a) * spec2


def spec_augment_lcg(spec: torch.Tensor, freq_mask_param: int, num_freq_masks: int, time_mask_param: int,
                     num_time_masks: int, seed: int) -> torch.Tensor:
    """SpecAugment on a [freq, time] spectrogram with the reference's draw order: state = seed +
    0xdeadbeef; per mask a length (state >> 32) % min(param, size) and a start (state >> 32) %
    max(size - length, 1), frequency masks first. A zero parameter draws no mask."""
    if spec.dim() != 2:
        raise ValueError("spec_augment requires a 2D [channels, frames] tensor")
    nf, nt = spec.shape
    state = (seed + 0xDEADBEEF) & _M64

    def draw():
        nonlocal state
        state = (state * _LCG_A + _LCG_C) & _M64
        return state >> 32

    for count, param, size, mask in ((num_freq_masks, freq_mask_param, nf, frequency_mask),
                                     (num_time_masks, time_mask_param, nt, time_mask_spec)):
        for _ in range(count):
            hi = min(param, size)
            if hi == 0:
                continue
            ln = draw() % hi
            st = draw() % max(size - ln, 1)
            mask(spec, st, ln)
    return spec


# ------------------------------------------------------------------------------------------ wavelets
@lru_cache(maxsize=None)
def daubechies_filter(taps: int) -> tuple:
    """Low-pass decomposition filter of the Daubechies wavelet with `taps` coefficients (taps / 2
    vanishing moments; 2 taps is Haar). Spectral factorisation: the half-band polynomial
    P(y) = sum_k C(N - 1 + k, k) y^k has roots y_k; each maps through y = (2 - z - 1/z) / 4 to a pair
    (z, 1/z), the root inside the unit circle goes into Q(z), and h = (1 + z)^N Q(z) scaled to sum sqrt(2),
    listed from the largest power down (the minimum-phase order)."""
    if taps < 2 or taps % 2:
        raise ValueError("a Daubechies filter has an even number of taps >= 2")
    n = taps // 2
    p = [math.comb(n - 1 + k, k) for k in range(n)]  # increasing powers of y
    poly = np.array([1.0])
    if n > 1:
        for yk in np.roots(p[::-1]):
            # z^2 - (2 - 4 y) z + 1 = 0
            zs = np.roots([1.0, -(2.0 - 4.0 * yk), 1.0])
            z = zs[np.argmin(np.abs(zs))]
            poly = np.convolve(poly, [1.0, -z])
    for _ in range(n):
        poly = np.convolve(poly, [1.0, 1.0])
    h = np.real(poly)
    h = h * (math.sqrt(2.0) / h.sum())
    return tuple(float(v) for v in h)


class WaveletType:
    HAAR, DB2, DB4, DB6, DB8 = 2, 4, 8, 12, 16  # number of filter taps

    @staticmethod
    def low_pass_filter(w: int) -> torch.Tensor:
        return torch.tensor(daubechies_filter(w), dtype=torch.float64)

    @staticmethod
    def high_pass_filter(w: int) -> torch.Tensor:
        """Quadrature mirror of the low-pass: h[i] = (-1)^(i+1) g[L - 1 - i]."""
        g = daubechies_filter(w)
        L = len(g)
        return torch.tensor([(1.0 if i % 2 else -1.0) * g[L - 1 - i] for i in range(L)], dtype=torch.float64)


def dwt(signal: torch.Tensor, wavelet: int = WaveletType.HAAR):
    """One level of the periodic DWT: approx[i] = sum_k x[(2i + k) mod n] g[k], detail likewise with the
    high-pass, for i < (n + L - 1) // 2. Returns (approx, detail) over the leading dimensions."""
    x = _f64(signal)
    n = x.shape[-1]
    if n == 0:
        raise ValueError("input signal cannot be empty")
    g, h = WaveletType.low_pass_filter(wavelet), WaveletType.high_pass_filter(wavelet)
    L = g.numel()
    m = (n + L - 1) // 2
    idx = (2 * torch.arange(m)[:, None] + torch.arange(L)[None, :]) % n  # [m, L]
    frames = x[..., idx.to(x.device)]  # [.., m, L]
    return frames @ g.to(x.device), frames @ h.to(x.device)


def idwt(approx: torch.Tensor, detail: torch.Tensor, wavelet: int = WaveletType.HAAR) -> torch.Tensor:
    """Periodic synthesis: out[(2i + k) mod 2m] += a[i] g[k] + d[i] h[k]."""
    a, d = _f64(approx), _f64(detail)
    if a.shape != d.shape:
        raise ValueError(f"idwt lengths differ: {tuple(a.shape)} vs {tuple(d.shape)}")
    g, h = WaveletType.low_pass_filter(wavelet).to(a.device), WaveletType.high_pass_filter(wavelet).to(a.device)
    m = a.shape[-1]
    L = g.numel()
    contrib = a[..., :, None] * g + d[..., :, None] * h  # [.., m, L]
    idx = ((2 * torch.arange(m)[:, None] + torch.arange(L)[None, :]) % (2 * m)).reshape(-1).to(a.device)
    out = torch.zeros(*a.shape[:-1], 2 * m, dtype=torch.float64, device=a.device)
    return out.index_add_(-1, idx, contrib.reshape(*a.shape[:-1], -1))


class WaveletDenoise:
    @staticmethod
    def soft_threshold(data: torch.Tensor, lam: float) -> torch.Tensor:
        """sign(x) max(|x| - lambda, 0)."""
        x = _f64(data)
        return torch.sign(x) * (x.abs() - lam).clamp_min(0.0)


# ------------------------------------------------------------------------------------------ codecs
_MU = 255.0
_A = 87.6


def mu_law_encode(signal: torch.Tensor) -> torch.Tensor:
    """8-bit mu-law (mu = 255): sign bit 0x80 for x >= 0, 7-bit round(127 ln(1 + mu|x|) / ln(1 + mu)),
    all bits inverted."""
    x = _f64(signal).clamp(-1.0, 1.0)
    q = torch.floor(torch.log1p(_MU * x.abs()) / math.log1p(_MU) * 127.0 + 0.5).to(torch.int64)
    code = torch.where(x < 0, q, q | 0x80)
    return (~code & 0xFF).to(torch.uint8)


def mu_law_decode(codes: torch.Tensor) -> torch.Tensor:
    inv = ~codes.to(torch.int64) & 0xFF
    sign = torch.where((inv & 0x80) != 0, 1.0, -1.0).to(torch.float64)
    y = (inv & 0x7F).to(torch.float64) / 127.0
    return sign * (torch.pow(1.0 + _MU, y) - 1.0) / _MU


def a_law_encode(signal: torch.Tensor) -> torch.Tensor:
    """8-bit A-law (A = 87.6): piecewise-linear below 1/A, logarithmic above; 7-bit magnitude, sign bit
    0x80 for x >= 0, even bits toggled (XOR 0x55)."""
    x = _f64(signal).clamp(-1.0, 1.0)
    m = x.abs()
    den = 1.0 + math.log(_A)
    comp = torch.where(m < 1.0 / _A, _A * m / den, (1.0 + torch.log(torch.clamp(_A * m, min=1e-300))) / den)
    q = torch.floor(comp * 127.0 + 0.5).to(torch.int64)
    code = torch.where(x < 0, q, q | 0x80)
    return (code ^ 0x55).to(torch.uint8)


def a_law_decode(codes: torch.Tensor) -> torch.Tensor:
    t = codes.to(torch.int64) ^ 0x55
    sign = torch.where((t & 0x80) != 0, 1.0, -1.0).to(torch.float64)
    y = (t & 0x7F).to(torch.float64) / 127.0
    den = 1.0 + math.log(_A)
    lin = torch.where(y < 1.0 / den, y * den / _A, torch.exp(y * den - 1.0) / _A)
    return sign * lin


def phonetic_one_hot(indices, vocab_size: int) -> torch.Tensor:
    """[vocab_size, seq_len] one-hot columns; an index >= vocab_size raises IndexError."""
    idx = torch.as_tensor(list(indices) if not torch.is_tensor(indices) else indices, dtype=torch.long)
    if idx.numel() and int(idx.max()) >= vocab_size:
        raise IndexError(f"phoneme index {int(idx.max())} outside vocabulary of {vocab_size}")
    out = torch.zeros(vocab_size, idx.numel(), dtype=torch.float64)
    out[idx, torch.arange(idx.numel())] = 1.0
    return out


# ------------------------------------------------------------------------------------------ frame features
def _frames(x: torch.Tensor, frame: int, hop: int) -> torch.Tensor:
    """[.., num_frames, frame] views with num_frames = (n - frame) // hop + 1 (0 when n < frame)."""
    if x.shape[-1] < frame or hop <= 0:
        return x.new_zeros(*x.shape[:-1], 0, frame)
    return x.unfold(-1, frame, hop)


def rms_frames(signal: torch.Tensor, frame_size: int, hop_size: int) -> torch.Tensor:
    f = _frames(_f64(signal), frame_size, hop_size)
    return f.square().mean(-1).sqrt() if f.shape[-2] else f.sum(-1)


def envelope_follower(signal: torch.Tensor, sample_rate: int, attack_ms: float, release_ms: float) -> torch.Tensor:
    """One-pole follower of |x| with separate coefficients exp(-1 / max(ms * sr / 1000, 1)) for rising
    (attack) and falling (release) input; one vector step per sample over the batch."""
    x = _f64(signal)
    ga = math.exp(-1.0 / max(attack_ms * 1e-3 * sample_rate, 1.0))
    gr = math.exp(-1.0 / max(release_ms * 1e-3 * sample_rate, 1.0))
    xs = x.reshape(-1, x.shape[-1]).abs().cpu().numpy()
    env = np.empty_like(xs)
    cur = np.zeros(xs.shape[0])
    for t in range(xs.shape[1]):
        tgt = xs[:, t]
        g = np.where(tgt > cur, ga, gr)
        cur = g * cur + (1.0 - g) * tgt
        env[:, t] = cur
    return torch.from_numpy(env).view_as(x).to(x.device)


def estimate_tempo(onset_envelope: torch.Tensor, hop_rate_hz: float, min_bpm: float = 60.0,
                   max_bpm: float = 200.0) -> float:
    """BPM of the autocorrelation peak of an onset envelope over lags [floor(60 r / max_bpm),
    min(ceil(60 r / min_bpm), n / 2)] (the first maximum wins); 120 for fewer than 32 frames."""
    e = _f64(onset_envelope).reshape(-1)
    n = e.numel()
    if n < 32:
        return 120.0
    lo = int(math.floor(hop_rate_hz * 60.0 / max_bpm))
    hi = min(int(math.ceil(hop_rate_hz * 60.0 / min_bpm)), n // 2)
    if hi < lo:
        return hop_rate_hz * 60.0 / max(lo, 1)
    lags = torch.arange(lo, hi + 1)
    corr = torch.stack([(e[: n - int(L)] * e[int(L):]).sum() for L in lags])
    best = int(lags[int(torch.argmax(corr))])
    return hop_rate_hz * 60.0 / max(best, 1) if best else math.inf


def pitch_autocorr(frame: torch.Tensor, sample_rate: int, min_f0: float, max_f0: float):
    """F0 from the normalised autocorrelation peak over lags [floor(sr / max_f0), min(ceil(sr / min_f0), n / 2)],
    refined by a parabola through the neighbours when the peak is interior; None when the peak
    correlation is at most 0.3 or the frame is shorter than 64 samples."""
    x = _f64(frame).reshape(-1)
    n = x.numel()
    if n < 64:
        return None
    lo = int(math.floor(sample_rate / max_f0))
    hi = int(math.ceil(sample_rate / min_f0))
    corrs = torch.zeros(hi + 2, dtype=torch.float64)
    best, best_c = 0, -math.inf
    for lag in range(lo, min(hi, n // 2) + 1):
        a, b = x[: n - lag], x[lag:]
        norm = math.sqrt(float(a @ a) * float(b @ b))
        c = float(a @ b) / norm if norm > 1e-10 else 0.0
        corrs[lag] = c
        if c > best_c:
            best_c, best = c, lag
    if best_c > 0.3 and lo < best < hi:
        al, be, ga = float(corrs[best - 1]), float(corrs[best]), float(corrs[best + 1])
        den = 2.0 * (2.0 * be - al - ga)
        delta = (ga - al) / den if abs(den) > 1e-9 else 0.0
        return sample_rate / (best + min(max(delta, -0.5), 0.5))
    if best_c > 0.3 and best > 0:
        return sample_rate / best
    return None


@dataclass
class VADConfig:
    frame_size: int = 512
    hop_size: int = 160
    threshold_db: float = -40.0
    min_speech_frames: int = 3
    min_silence_frames: int = 10


def compute_vad(signal: torch.Tensor, config: VADConfig | None = None) -> torch.Tensor:
    """Per-frame speech flags: frame energy (mean square) above 10^(dB/10), then hysteresis: speech
    starts after min_speech_frames active frames in a row and ends after min_silence_frames inactive
    ones. Leading dimensions are independent signals."""
    cfg = config or VADConfig()
    x = _f64(signal)
    f = _frames(x, cfg.frame_size, cfg.hop_size)
    raw = f.square().mean(-1) > 10.0 ** (cfg.threshold_db / 10.0)
    r = raw.reshape(-1, raw.shape[-1]).cpu().numpy()
    out = np.zeros_like(r)
    sp = np.zeros(r.shape[0], dtype=np.int64)
    si = np.zeros(r.shape[0], dtype=np.int64)
    state = np.zeros(r.shape[0], dtype=bool)
    for t in range(r.shape[1]):
        a = r[:, t]
        sp = np.where(a, sp + 1, 0)
        si = np.where(a, 0, si + 1)
        state = np.where(a & (sp >= cfg.min_speech_frames), True, state)
        state = np.where(~a & (si >= cfg.min_silence_frames), False, state)
        out[:, t] = state
    return torch.from_numpy(out).view(raw.shape)


def trim_silence(signal: torch.Tensor, threshold_db: float = -40.0, frame_size: int = 512,
                 hop_size: int = 160) -> torch.Tensor:
    """Cut leading and trailing frames whose energy is at or below the threshold (a 1-D signal, or
    [channels, n] judged on the channel mean); unchanged when nothing would remain."""
    x = _f64(signal)
    mono = x if x.dim() == 1 else x.mean(0)
    n = mono.numel()
    if n < frame_size:
        return x.clone()
    active = (_frames(mono, frame_size, hop_size).square().mean(-1) > 10.0 ** (threshold_db / 10.0)).tolist()
    nf = len(active)
    s = next((i for i in range(nf) if active[i]), nf)
    e = nf
    while e > s and not active[e - 1]:
        e -= 1
    a, b = s * hop_size, min(e * hop_size + frame_size, n)
    return x.clone() if a >= b else x[..., a:b].clone()


# ------------------------------------------------------------------ the reference's remaining names
# crates/brain-audio/src: features.rs (amplitude/power <-> dB), window.rs (Bartlett, Blackman), scales.rs
# (ERB), analysis.rs (Hilbert envelope, real cepstrum), vocoder.rs (PhaseVocoder), distance.rs
# (vector_distance with a DistanceMetric), config.rs (MelConfig presets default_speech / default_music),
# util.rs (samples_from_duration, ensure_length, nyquist_hz, fft_freqs), preprocess.rs (de_emphasis).

def amplitude_to_db(x: torch.Tensor, amin: float = 1e-10, top_db: float | None = None) -> torch.Tensor:
    d = 20.0 * torch.log10(x.abs().clamp_min(amin))
    return torch.maximum(d, d.max() - top_db) if top_db is not None else d


def power_to_db(x: torch.Tensor, amin: float = 1e-10, top_db: float | None = None) -> torch.Tensor:
    d = 10.0 * torch.log10(x.clamp_min(amin))
    return torch.maximum(d, d.max() - top_db) if top_db is not None else d


def db_to_amplitude(d: torch.Tensor) -> torch.Tensor:
    return torch.pow(10.0, d / 20.0)


def db_to_power(d: torch.Tensor) -> torch.Tensor:
    return torch.pow(10.0, d / 10.0)


def bartlett_window(n: int, periodic: bool = True, dtype=torch.float32) -> torch.Tensor:
    return torch.bartlett_window(n, periodic=periodic, dtype=dtype)


def blackman_window(n: int, periodic: bool = True, dtype=torch.float32) -> torch.Tensor:
    return torch.blackman_window(n, periodic=periodic, dtype=dtype)


def hz_to_erb(f):
    """Glasberg & Moore (1990) ERB-rate scale: 21.4 log10(1 + 0.00437 f)."""
    f = torch.as_tensor(f, dtype=torch.float64)
    return 21.4 * torch.log10(1.0 + 0.00437 * f)


def erb_to_hz(e):
    e = torch.as_tensor(e, dtype=torch.float64)
    return (torch.pow(10.0, e / 21.4) - 1.0) / 0.00437


def hilbert_envelope(x: torch.Tensor) -> torch.Tensor:
    """|analytic signal| along the last axis (FFT, doubled positive frequencies, zeroed negative ones)."""
    n = x.shape[-1]
    X = torch.fft.fft(x.double(), dim=-1)
    h = torch.zeros(n, dtype=torch.float64, device=x.device)
    h[0] = 1.0
    if n % 2 == 0:
        h[n // 2] = 1.0
        h[1:n // 2] = 2.0
    else:
        h[1:(n + 1) // 2] = 2.0
    return torch.fft.ifft(X * h, dim=-1).abs().to(x.dtype)


def real_cepstrum(x: torch.Tensor, eps: float = 1e-12) -> torch.Tensor:
    return torch.fft.ifft(torch.log(torch.fft.fft(x.double(), dim=-1).abs().clamp_min(eps)), dim=-1).real.to(x.dtype)


def de_emphasis(x: torch.Tensor, coef: float = 0.97) -> torch.Tensor:
    """Inverse of pre-emphasis: y[n] = x[n] + coef y[n-1]."""
    y = torch.empty_like(x)
    acc = torch.zeros_like(x[..., 0])
    for i in range(x.shape[-1]):
        acc = x[..., i] + coef * acc
        y[..., i] = acc
    return y


def samples_from_duration(seconds: float, sample_rate: int) -> int:
    return int(round(seconds * sample_rate))


def nyquist_hz(sample_rate: int) -> float:
    return sample_rate / 2.0


def fft_freqs(n_fft: int, sample_rate: int) -> torch.Tensor:
    return torch.fft.rfftfreq(n_fft, 1.0 / sample_rate)


def ensure_length(x: torch.Tensor, n: int) -> torch.Tensor:
    """Zero-pad or cut the last axis to n samples."""
    if x.shape[-1] >= n:
        return x[..., :n]
    return torch.nn.functional.pad(x, (0, n - x.shape[-1]))


class DistanceMetric:
    EUCLIDEAN, COSINE, MANHATTAN = "euclidean", "cosine", "manhattan"


def vector_distance(a: torch.Tensor, b: torch.Tensor, metric: str = "euclidean") -> float:
    a, b = a.double().reshape(-1), b.double().reshape(-1)
    if metric == "euclidean":
        return float((a - b).norm())
    if metric == "manhattan":
        return float((a - b).abs().sum())
    if metric == "cosine":
        d = a.norm() * b.norm()
        return float(1.0 - a @ b / d) if d > 0 else 1.0
    raise ValueError(f"unknown distance {metric!r}")


class PhaseVocoder:
    """Time-scale modification in the STFT domain (Flanagan & Golden; Laroche & Dolson phase propagation):
    frames are read at ``rate`` times the hop, magnitudes interpolated and phases advanced by the
    measured instantaneous frequency."""

    def __init__(self, n_fft: int = 1024, hop: int = 256):
        self.n_fft, self.hop = n_fft, hop

    def stretch(self, x: torch.Tensor, rate: float) -> torch.Tensor:
        win = torch.hann_window(self.n_fft, dtype=torch.float64)
        S = torch.stft(x.double(), self.n_fft, self.hop, window=win, return_complex=True)  # [F, T]
        F_, T = S.shape
        steps = torch.arange(0, T - 1, rate, dtype=torch.float64)
        omega = torch.linspace(0, torch.pi * self.hop, F_, dtype=torch.float64)
        phase = torch.angle(S[:, 0])
        out = torch.empty(F_, len(steps), dtype=torch.complex128)
        for k, t in enumerate(steps):
            i = int(t)
            frac = float(t - i)
            a, b = S[:, i], S[:, i + 1]
            mag = (1 - frac) * a.abs() + frac * b.abs()
            out[:, k] = torch.polar(mag, phase)
            dphi = torch.angle(b) - torch.angle(a) - omega
            dphi = dphi - 2 * torch.pi * torch.round(dphi / (2 * torch.pi))
            phase = phase + omega + dphi
        y = torch.istft(out, self.n_fft, self.hop, window=win, length=int(round(x.shape[-1] / rate)))
        return y.to(x.dtype)


@dataclass
class MelConfig:
    sample_rate: int = 16000
    n_fft: int = 400
    hop_length: int = 160
    n_mels: int = 80
    f_min: float = 0.0
    f_max: float | None = None

    @classmethod
    def default_speech(cls) -> "MelConfig":
        return cls(16000, 400, 160, 80)

    @classmethod
    def default_speech_80(cls) -> "MelConfig":
        return cls.default_speech()

    @classmethod
    def default_music(cls) -> "MelConfig":
        return cls(22050, 2048, 512, 128)

    @classmethod
    def default_music_128(cls) -> "MelConfig":
        return cls.default_music()
