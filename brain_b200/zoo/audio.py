"""Audio features: framing and windows, STFT / inverse STFT, mel filterbank, log-mel spectrogram, MFCC
(DCT-II), CMVN, pre-emphasis, energy-based voice activity detection, resampling, SpecAugment masks and
16-bit PCM WAV read / write.

Reference: crates/brain-audio. STFT (feature/stft.rs:14-220), MFCC (feature/mfcc.rs:13-160 incl. CMVN
at :96), spectral augmentation (augment/spectral.rs), time augmentation (augment/time.rs), VAD
(vad.rs), resampling (resample.rs), WAV I/O (io/wav.rs).

Batched tensor code: the STFT is ``torch.stft`` (one cuFFT batch on a GPU), the mel projection and the
DCT are GEMMs against precomputed matrices. Mel scale is HTK (2595 log10(1 + f / 700)).
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass

import torch


@dataclass
class STFTConfig:
    n_fft: int = 512
    hop_length: int = 160
    win_length: int = 400
    window: str = "hann"
    center: bool = True


def _window(cfg: STFTConfig, device=None, dtype=torch.float32):
    if cfg.window == "hann":
        return torch.hann_window(cfg.win_length, periodic=True, device=device, dtype=dtype)
    if cfg.window == "hamming":
        return torch.hamming_window(cfg.win_length, periodic=True, device=device, dtype=dtype)
    return torch.ones(cfg.win_length, device=device, dtype=dtype)


def stft(signal: torch.Tensor, cfg: STFTConfig | None = None):
    """signal [..., n] -> (magnitude, phase), each [..., n_fft // 2 + 1, frames]."""
    cfg = cfg or STFTConfig()
    spec = torch.stft(signal, cfg.n_fft, cfg.hop_length, cfg.win_length, _window(cfg, signal.device, signal.dtype),
                      center=cfg.center, return_complex=True)
    return spec.abs(), spec.angle()


def istft(magnitude, phase, cfg: STFTConfig | None = None, length: int | None = None):
    cfg = cfg or STFTConfig()
    spec = torch.polar(magnitude, phase)
    return torch.istft(spec, cfg.n_fft, cfg.hop_length, cfg.win_length, _window(cfg, magnitude.device, magnitude.dtype),
                       center=cfg.center, length=length)


def hz_to_mel(f):
    return 2595.0 * torch.log10(1.0 + torch.as_tensor(f, dtype=torch.float64) / 700.0)


def mel_to_hz(m):
    return 700.0 * (10.0 ** (torch.as_tensor(m, dtype=torch.float64) / 2595.0) - 1.0)


def mel_filterbank(n_mels: int, n_fft: int, sample_rate: int, f_min: float = 0.0, f_max: float | None = None):
    """Triangular filters [n_mels, n_fft // 2 + 1] evenly spaced on the mel scale."""
    f_max = f_max or sample_rate / 2
    mels = torch.linspace(float(hz_to_mel(f_min)), float(hz_to_mel(f_max)), n_mels + 2, dtype=torch.float64)
    hz = mel_to_hz(mels)
    bins = torch.linspace(0, sample_rate / 2, n_fft // 2 + 1, dtype=torch.float64)
    fb = torch.zeros(n_mels, bins.numel(), dtype=torch.float64)
    for m in range(n_mels):
        lo, c, hi = hz[m], hz[m + 1], hz[m + 2]
        up = (bins - lo) / (c - lo)
        down = (hi - bins) / (hi - c)
        fb[m] = torch.clamp(torch.minimum(up, down), min=0)
    return fb.float()


def dct_matrix(n_out: int, n_in: int) -> torch.Tensor:
    """Orthonormal DCT-II [n_out, n_in]."""
    k = torch.arange(n_out, dtype=torch.float64)[:, None]
    n = torch.arange(n_in, dtype=torch.float64)[None]
    m = torch.cos(math.pi / n_in * (n + 0.5) * k) * math.sqrt(2.0 / n_in)
    m[0] /= math.sqrt(2.0)
    return m.float()


@dataclass
class MFCCConfig:
    sample_rate: int = 16000
    n_mfcc: int = 13
    n_mels: int = 40
    stft: STFTConfig = None
    log_eps: float = 1e-10

    def __post_init__(self):
        if self.stft is None:
            self.stft = STFTConfig()


def log_mel_spectrogram(signal, cfg: MFCCConfig | None = None):
    """[..., n] -> [..., n_mels, frames] natural-log mel power."""
    cfg = cfg or MFCCConfig()
    mag, _ = stft(signal, cfg.stft)
    fb = mel_filterbank(cfg.n_mels, cfg.stft.n_fft, cfg.sample_rate).to(signal.device, mag.dtype)
    return torch.log(torch.matmul(fb, mag ** 2) + cfg.log_eps)


def mfcc(signal, cfg: MFCCConfig | None = None):
    cfg = cfg or MFCCConfig()
    lm = log_mel_spectrogram(signal, cfg)
    return torch.matmul(dct_matrix(cfg.n_mfcc, cfg.n_mels).to(lm.device, lm.dtype), lm)


def apply_cmvn(features, norm_mean: bool = True, norm_var: bool = True, dim: int = -1):
    """Cepstral mean (and variance) normalisation along the time axis."""
    out = features
    if norm_mean:
        out = out - out.mean(dim, keepdim=True)
    if norm_var:
        out = out / (out.std(dim, keepdim=True, unbiased=False) + 1e-8)
    return out


def pre_emphasis(signal, coef: float = 0.97):
    return torch.cat([signal[..., :1], signal[..., 1:] - coef * signal[..., :-1]], -1)


def frame_energy(signal, frame: int = 400, hop: int = 160):
    frames = signal.unfold(-1, frame, hop)
    return (frames ** 2).mean(-1)


def energy_vad(signal, frame: int = 400, hop: int = 160, threshold_db: float = -35.0):
    """True per frame whose energy is within ``threshold_db`` of the loudest frame."""
    e = frame_energy(signal, frame, hop)
    db = 10 * torch.log10(e + 1e-12)
    return db > (db.max(-1, keepdim=True).values + threshold_db)


def resample(signal, orig_sr: int, new_sr: int):
    """Band-limited resampling via linear interpolation after a windowed-sinc low-pass when downsampling."""
    if orig_sr == new_sr:
        return signal
    x = signal
    if new_sr < orig_sr:
        cutoff = new_sr / orig_sr / 2
        half = 32
        n = torch.arange(-half, half + 1, dtype=torch.float64)
        h = 2 * cutoff * torch.sinc(2 * cutoff * n) * torch.hann_window(2 * half + 1, periodic=False, dtype=torch.float64)
        h = (h / h.sum()).to(x.dtype).to(x.device)
        x = torch.nn.functional.conv1d(x.reshape(-1, 1, x.shape[-1]), h.view(1, 1, -1), padding=half).reshape(x.shape)
    n_out = int(round(x.shape[-1] * new_sr / orig_sr))
    return torch.nn.functional.interpolate(x.reshape(-1, 1, x.shape[-1]), size=n_out, mode="linear",
                                           align_corners=False).reshape(*x.shape[:-1], n_out)


def spec_augment(spec, freq_mask: int = 8, time_mask: int = 20, n_freq: int = 1, n_time: int = 1, generator=None):
    """Zeroes ``n_freq`` random frequency bands and ``n_time`` random time spans of [..., F, T]."""
    out = spec.clone()
    F_, T_ = spec.shape[-2], spec.shape[-1]
    for _ in range(n_freq):
        w = int(torch.randint(0, freq_mask + 1, (1,), generator=generator))
        f0 = int(torch.randint(0, max(1, F_ - w), (1,), generator=generator))
        out[..., f0:f0 + w, :] = 0
    for _ in range(n_time):
        w = int(torch.randint(0, time_mask + 1, (1,), generator=generator))
        t0 = int(torch.randint(0, max(1, T_ - w), (1,), generator=generator))
        out[..., :, t0:t0 + w] = 0
    return out


def write_wav(path: str, samples: torch.Tensor, sample_rate: int) -> None:
    """Mono or [channels, n] float samples in [-1, 1] -> 16-bit PCM RIFF/WAVE."""
    x = samples if samples.dim() == 2 else samples[None]
    ch, n = x.shape
    pcm = (x.clamp(-1, 1) * 32767).round().to(torch.int16).t().contiguous().numpy().tobytes()
    with open(path, "wb") as f:
        f.write(b"RIFF" + struct.pack("<I", 36 + len(pcm)) + b"WAVE")
        f.write(b"fmt " + struct.pack("<IHHIIHH", 16, 1, ch, sample_rate, sample_rate * ch * 2, ch * 2, 16))
        f.write(b"data" + struct.pack("<I", len(pcm)) + pcm)


def read_wav(path: str):
    """16-bit PCM WAV -> (float samples [channels, n], sample_rate)."""
    import numpy as np

    with open(path, "rb") as f:
        data = f.read()
    if data[:4] != b"RIFF" or data[8:12] != b"WAVE":
        raise ValueError("not a RIFF/WAVE file")
    pos, fmt, pcm = 12, None, None
    while pos + 8 <= len(data):
        cid, size = data[pos:pos + 4], struct.unpack("<I", data[pos + 4:pos + 8])[0]
        body = data[pos + 8:pos + 8 + size]
        if cid == b"fmt ":
            fmt = struct.unpack("<HHIIHH", body[:16])
        elif cid == b"data":
            pcm = body
        pos += 8 + size + (size & 1)
    if fmt is None or pcm is None or fmt[0] != 1 or fmt[5] != 16:
        raise ValueError("only 16-bit PCM WAV is supported")
    ch, sr = fmt[1], fmt[2]
    x = torch.from_numpy(np.frombuffer(pcm, dtype="<i2").astype("float32") / 32768.0)
    return x.view(-1, ch).t().contiguous(), sr


def dtw(a: torch.Tensor, b: torch.Tensor):
    """Dynamic time warping between feature sequences a [N, F] and b [M, F] with Euclidean local cost:
    returns (total cost, alignment path as (i, j) pairs). Reference: align.rs."""
    cost = torch.cdist(a.double().reshape(a.shape[0], -1), b.double().reshape(b.shape[0], -1))
    N, M = cost.shape
    D = torch.full((N + 1, M + 1), float("inf"), dtype=torch.float64)
    D[0, 0] = 0.0
    for i in range(1, N + 1):
        for j in range(1, M + 1):
            D[i, j] = cost[i - 1, j - 1] + min(D[i - 1, j], D[i, j - 1], D[i - 1, j - 1])
    path, i, j = [], N, M
    while i > 0 and j > 0:
        path.append((i - 1, j - 1))
        step = int(torch.argmin(torch.stack([D[i - 1, j - 1], D[i - 1, j], D[i, j - 1]])))
        i, j = (i - 1, j - 1) if step == 0 else ((i - 1, j) if step == 1 else (i, j - 1))
    return float(D[N, M]), path[::-1]


def yin_pitch(frame: torch.Tensor, sample_rate: int, fmin: float = 50.0, fmax: float = 1000.0,
              threshold: float = 0.1) -> float:
    """Fundamental frequency of one frame by the YIN method (de Cheveigné and Kawahara 2002):
    cumulative-mean-normalised difference function, first dip below ``threshold``, parabolic
    interpolation. Returns 0.0 for an unvoiced frame. Reference: features_pitch.rs."""
    x = frame.double()
    tmin, tmax = int(sample_rate / fmax), min(int(sample_rate / fmin), x.numel() // 2)
    if tmax <= tmin + 1 or float((x * x).mean()) < 1e-12:  # too short, or silence
        return 0.0
    W = x.numel() - tmax
    d = torch.stack([((x[:W] - x[t:t + W]) ** 2).sum() for t in range(tmax + 1)])
    cmnd = torch.ones_like(d)
    cum = torch.cumsum(d[1:], 0)
    cmnd[1:] = d[1:] * torch.arange(1, tmax + 1, dtype=torch.float64) / cum.clamp_min(1e-12)
    tau = None
    for t in range(tmin, tmax):
        if cmnd[t] < threshold:
            while t + 1 < tmax and cmnd[t + 1] < cmnd[t]:
                t += 1
            tau = t
            break
    if tau is None:
        return 0.0
    if 0 < tau < tmax:
        a, b, c = float(cmnd[tau - 1]), float(cmnd[tau]), float(cmnd[tau + 1])
        den = a - 2 * b + c
        shift = 0.5 * (a - c) / den if abs(den) > 1e-12 else 0.0
    else:
        shift = 0.0
    return sample_rate / (tau + shift)


def chroma(signal: torch.Tensor, sample_rate: int, cfg: STFTConfig | None = None, n_chroma: int = 12) -> torch.Tensor:
    """Pitch-class energy [12, frames]: every STFT bin above 20 Hz is assigned to the nearest equal-
    tempered pitch class (A4 = 440 Hz), columns normalised to unit maximum. Reference: feature/tonal.rs."""
    cfg = cfg or STFTConfig()
    mag, _ = stft(signal, cfg)
    freqs = torch.linspace(0, sample_rate / 2, mag.shape[-2])
    valid = freqs > 20
    pc = torch.zeros(mag.shape[-2], dtype=torch.long)
    pc[valid] = (torch.round(12 * torch.log2(freqs[valid] / 440.0)).long() + 9) % n_chroma  # 0 = C
    out = torch.zeros(n_chroma, mag.shape[-1])
    out.index_add_(0, pc[valid], (mag[valid] ** 2).float())
    return out / out.amax(0, keepdim=True).clamp_min(1e-12)


# --------------------------------------------------------------------------- denoising
def spectral_subtraction(signal: torch.Tensor, cfg: STFTConfig | None = None, oversubtraction: float = 1.0,
                         spectral_floor: float = 0.01, noise_frames: int = 5) -> torch.Tensor:
    """Spectral subtraction (Boll 1979; crates/brain-audio/src/denoise.rs:13-62): the noise power per
    frequency bin is the mean over the first ``noise_frames`` frames; each bin keeps
    sqrt(max(|X|^2 - oversubtraction * noise, spectral_floor * |X|^2)) with the noisy phase; the inverse
    STFT restores the original length."""
    cfg = cfg or STFTConfig()
    mag, phase = stft(signal, cfg)
    power = mag ** 2
    noise = power[..., : min(noise_frames, power.shape[-1])].mean(-1, keepdim=True)
    clean = torch.sqrt(torch.maximum(power - oversubtraction * noise, spectral_floor * power))
    return istft(clean, phase, cfg, length=signal.shape[-1])


def minimum_statistics_noise(power: torch.Tensor, window: int = 50, smoothing: float = 0.8) -> torch.Tensor:
    """Stationary noise-floor estimate by minimum statistics (Martin 2001, simplified): the power
    spectrum [.., bins, frames] is smoothed recursively over time and the noise floor of each frame is
    the minimum of the smoothed power over the last ``window`` frames."""
    sm = power.clone()
    for t in range(1, power.shape[-1]):
        sm[..., t] = smoothing * sm[..., t - 1] + (1 - smoothing) * power[..., t]
    pad = torch.nn.functional.pad(sm, (window - 1, 0), value=float("inf"))
    return -torch.nn.functional.max_pool1d(-pad.reshape(-1, 1, pad.shape[-1]), window, 1).reshape(sm.shape)


def wiener_filter(signal: torch.Tensor, cfg: STFTConfig | None = None, noise_frames: int = 5, dd_alpha: float = 0.98,
                  gain_floor: float = 0.05, min_stats: bool = False) -> torch.Tensor:
    """Wiener filtering with the decision-directed a-priori SNR estimate (Ephraim and Malah 1984):
    xi_t = a G_{t-1}^2 |X_{t-1}|^2 / N + (1 - a) max(|X_t|^2 / N - 1, 0), gain G = xi / (1 + xi)
    (floored). The noise power N comes from the first frames, or from minimum statistics per frame."""
    cfg = cfg or STFTConfig()
    mag, phase = stft(signal, cfg)
    power = mag ** 2
    if min_stats:
        noise = minimum_statistics_noise(power).clamp_min(1e-12)
    else:
        noise = power[..., : min(noise_frames, power.shape[-1])].mean(-1, keepdim=True).clamp_min(1e-12)
        noise = noise.expand_as(power)
    gains = torch.empty_like(power)
    prev = torch.zeros_like(power[..., 0])
    for t in range(power.shape[-1]):
        post = power[..., t] / noise[..., t]
        xi = dd_alpha * prev / noise[..., t] + (1 - dd_alpha) * (post - 1).clamp_min(0)
        g = (xi / (1 + xi)).clamp_min(gain_floor)
        gains[..., t] = g
        prev = (g ** 2) * power[..., t]
    return istft(mag * gains, phase, cfg, length=signal.shape[-1])


def snr_db(clean: torch.Tensor, estimate: torch.Tensor) -> float:
    """10 log10(|clean|^2 / |clean - estimate|^2)."""
    err = (clean - estimate).pow(2).sum().clamp_min(1e-30)
    return float(10 * torch.log10(clean.pow(2).sum() / err))
