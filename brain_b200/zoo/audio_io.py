"""Audio containers and descriptors: a multi-channel ``AudioBuffer``, FLAC STREAMINFO and MPEG audio frame
header parsing, mel/Bark scale conversions, delta features, spectral descriptors, zero-crossing rate and
CENS chroma.

Reference: crates/brain-audio/src/core.rs (SampleRate, Channels, AudioBuffer), io/flac.rs
(parse_flac_metadata), io/mp3.rs (Mp3FrameHeader, parse_mp3_frames), utils.rs (Slaney / HTK mel, Bark),
feature/spectral.rs (compute_deltas, SpectralDescriptors), feature/tonal.rs (zero_crossing_rate,
spectral_flux, chroma_cens). The MPEG parser covers MPEG-1, -2 and -2.5, layers I-III with the
standard bitrate and sample-rate tables and frame-length rules (ISO/IEC 11172-3, 13818-3); the
reference reads every header with the MPEG-1 layer III table. Spectral descriptors take [bins, frames]
magnitudes (optionally with leading batch dimensions) and work on all frames at once.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


# ------------------------------------------------------------------------------------------ buffers
class AudioBuffer:
    """Samples as a [channels, samples] float64 tensor with a sample rate."""

    def __init__(self, samples: torch.Tensor, sample_rate: int):
        s = torch.as_tensor(samples, dtype=torch.float64)
        self.data = s[None] if s.dim() == 1 else s
        if sample_rate <= 0:
            raise ValueError("sample rate must be positive")
        self.sample_rate = int(sample_rate)

    @classmethod
    def zeros(cls, channels: int, num_samples: int, sample_rate: int) -> "AudioBuffer":
        return cls(torch.zeros(channels, num_samples, dtype=torch.float64), sample_rate)

    @property
    def channels(self) -> int:
        return self.data.shape[0]

    @property
    def num_samples(self) -> int:
        return self.data.shape[1]

    def duration(self) -> float:
        return self.num_samples / self.sample_rate

    def channel(self, ch: int) -> torch.Tensor:
        if not 0 <= ch < self.channels:
            raise IndexError(f"channel {ch} of {self.channels}")
        return self.data[ch]

    def slice(self, start: int, end: int) -> "AudioBuffer":
        if not 0 <= start <= end <= self.num_samples:
            raise ValueError(f"slice [{start}, {end}) outside {self.num_samples} samples")
        return AudioBuffer(self.data[:, start:end].clone(), self.sample_rate)

    def to_mono(self) -> "AudioBuffer":
        return AudioBuffer(self.data.mean(0, keepdim=True), self.sample_rate)

    def to_stereo(self) -> "AudioBuffer":
        if self.channels == 2:
            return AudioBuffer(self.data.clone(), self.sample_rate)
        if self.channels != 1:
            raise ValueError("only mono converts to stereo")
        return AudioBuffer(self.data.repeat(2, 1), self.sample_rate)

    def concat(self, other: "AudioBuffer") -> "AudioBuffer":
        if other.channels != self.channels or other.sample_rate != self.sample_rate:
            raise ValueError("concat needs equal channel counts and sample rates")
        return AudioBuffer(torch.cat([self.data, other.data], 1), self.sample_rate)

    def mix(self, other: "AudioBuffer", weight: float) -> None:
        """self += weight * other over the common length."""
        if other.channels != self.channels:
            raise ValueError("mix needs equal channel counts")
        n = min(self.num_samples, other.num_samples)
        self.data[:, :n] += weight * other.data[:, :n]

    def scale(self, factor: float) -> None:
        self.data *= factor

    def peak_amplitude(self) -> float:
        return float(self.data.abs().max()) if self.data.numel() else 0.0

    def normalize_peak(self, target_peak: float = 1.0) -> None:
        p = self.peak_amplitude()
        if p > 0:
            self.data *= target_peak / p

    def rms_energy(self) -> float:
        return float(self.data.square().mean().sqrt()) if self.data.numel() else 0.0


# ------------------------------------------------------------------------------------------ containers
@dataclass
class FlacStreamInfo:
    min_block_size: int
    max_block_size: int
    min_frame_size: int
    max_frame_size: int
    sample_rate: int
    channels: int
    bits_per_sample: int
    total_samples: int


def parse_flac_metadata(data: bytes) -> FlacStreamInfo:
    """The STREAMINFO block that must follow the "fLaC" marker: big-endian block sizes (16 bit), frame sizes
    (24 bit), then a 64-bit word holding sample rate (20 bits), channels - 1 (3), bits per sample - 1 (5)
    and total samples (36)."""
    if len(data) < 42:
        raise ValueError("FLAC stream shorter than the minimum header")
    if data[:4] != b"fLaC":
        raise ValueError("invalid FLAC marker")
    if data[4] & 0x7F != 0:
        raise ValueError("the first FLAC metadata block must be STREAMINFO")
    b = data[8:42]
    word = int.from_bytes(b[10:18], "big")
    return FlacStreamInfo(int.from_bytes(b[0:2], "big"), int.from_bytes(b[2:4], "big"), int.from_bytes(b[4:7], "big"),
                          int.from_bytes(b[7:10], "big"), word >> 44, ((word >> 41) & 0x7) + 1,
                          ((word >> 36) & 0x1F) + 1, word & ((1 << 36) - 1))


_BITRATES = {  # kbit/s by (MPEG-1?, layer); index 1..14
    (True, 1): [32, 64, 96, 128, 160, 192, 224, 256, 288, 320, 352, 384, 416, 448],
    (True, 2): [32, 48, 56, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384],
    (True, 3): [32, 40, 48, 56, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320],
    (False, 1): [32, 48, 56, 64, 80, 96, 112, 128, 144, 160, 176, 192, 224, 256],
    (False, 2): [8, 16, 24, 32, 40, 48, 56, 64, 80, 96, 112, 128, 144, 160],
}
_BITRATES[(False, 3)] = _BITRATES[(False, 2)]
_RATES = {1: (44100, 48000, 32000), 2: (22050, 24000, 16000), 25: (11025, 12000, 8000)}


@dataclass
class Mp3FrameHeader:
    version: int  # 1, 2 or 25 (MPEG-2.5)
    layer: int
    bitrate_kbps: int
    sample_rate: int
    padding: bool
    channels: int
    frame_size: int

    @classmethod
    def parse(cls, h: bytes) -> "Mp3FrameHeader":
        if len(h) < 4 or h[0] != 0xFF or (h[1] & 0xE0) != 0xE0:
            raise ValueError("invalid MPEG audio sync word")
        version = {3: 1, 2: 2, 0: 25}.get((h[1] >> 3) & 0x3)
        layer = {3: 1, 2: 2, 1: 3}.get((h[1] >> 1) & 0x3)
        if version is None or layer is None:
            raise ValueError("reserved MPEG version or layer")
        bi, si = (h[2] >> 4) & 0xF, (h[2] >> 2) & 0x3
        if bi in (0, 15) or si == 3:
            raise ValueError("free-format or invalid bitrate / sample-rate index")
        br = _BITRATES[(version == 1, layer)][bi - 1]
        sr = _RATES[version][si]
        pad = bool((h[2] >> 1) & 1)
        if layer == 1:
            size = (12 * br * 1000 // sr + pad) * 4
        else:
            size = (144 if (layer == 2 or version == 1) else 72) * br * 1000 // sr + pad
        return cls(version, layer, br, sr, pad, 1 if (h[3] >> 6) == 3 else 2, size)


def parse_mp3_frames(data: bytes) -> list:
    """Walk the stream: at every sync word that parses, record the header and jump one frame; else step
    one byte."""
    out, i = [], 0
    while i + 4 <= len(data):
        if data[i] == 0xFF and (data[i + 1] & 0xE0) == 0xE0:
            try:
                hdr = Mp3FrameHeader.parse(data[i:i + 4])
                out.append(hdr)
                i += max(hdr.frame_size, 4)
                continue
            except ValueError:
                pass
        i += 1
    return out


# ------------------------------------------------------------------------------------------ scales
def hz_to_mel_htk(hz):
    return 2595.0 * torch.log10(1.0 + torch.as_tensor(hz, dtype=torch.float64) / 700.0)


def mel_to_hz_htk(mel):
    return 700.0 * (10.0 ** (torch.as_tensor(mel, dtype=torch.float64) / 2595.0) - 1.0)


_F_SP, _MIN_LOG_HZ = 200.0 / 3, 1000.0
_MIN_LOG_MEL = _MIN_LOG_HZ / _F_SP
_LOGSTEP = math.log(6.4) / 27.0


def hz_to_mel_slaney(hz):
    """Slaney's scale: linear (200/3 Hz per mel) below 1 kHz, logarithmic above."""
    f = torch.as_tensor(hz, dtype=torch.float64)
    return torch.where(f >= _MIN_LOG_HZ, _MIN_LOG_MEL + torch.log(f.clamp_min(1e-300) / _MIN_LOG_HZ) / _LOGSTEP,
                       f / _F_SP)


def mel_to_hz_slaney(mel):
    m = torch.as_tensor(mel, dtype=torch.float64)
    return torch.where(m >= _MIN_LOG_MEL, _MIN_LOG_HZ * torch.exp(_LOGSTEP * (m - _MIN_LOG_MEL)), m * _F_SP)


def hz_to_bark(hz):
    """Traunmueller 1990: 26.81 f / (1960 + f) - 0.53."""
    f = torch.as_tensor(hz, dtype=torch.float64)
    return 26.81 * f / (1960.0 + f) - 0.53


def bark_to_hz(bark):
    z = torch.as_tensor(bark, dtype=torch.float64)
    return 1960.0 * (z + 0.53) / (26.28 - z)


# ------------------------------------------------------------------------------------------ features
def compute_deltas(features: torch.Tensor, order: int = 1, width: int = 9) -> torch.Tensor:
    """Regression deltas over frames (last dimension) with edge replication:
    d_t = sum_{k=1..N} k (c_{t+k} - c_{t-k}) / (2 sum k^2), N = max(width, 3) // 2; applied ``order`` times."""
    x = torch.as_tensor(features, dtype=torch.float64)
    n = max(width, 3) // 2
    T = x.shape[-1]
    den = 2.0 * sum(k * k for k in range(1, n + 1))
    t = torch.arange(T)
    for _ in range(order):
        num = torch.zeros_like(x)
        for k in range(1, n + 1):
            num += k * (x[..., (t + k).clamp(max=T - 1)] - x[..., (t - k).clamp(min=0)])
        x = num / den
    return x


class SpectralDescriptors:
    """Per-frame descriptors of magnitude spectra [..., bins, frames] with bin frequencies ``freqs``."""

    @staticmethod
    def spectral_centroid(mag: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
        m = mag.double()
        f = torch.as_tensor(freqs, dtype=torch.float64)[:, None]
        den = m.sum(-2)
        return torch.where(den > 1e-12, (f * m).sum(-2) / den.clamp_min(1e-300), torch.zeros_like(den))

    @staticmethod
    def spectral_bandwidth(mag, freqs, p: float = 2.0) -> torch.Tensor:
        m = mag.double()
        f = torch.as_tensor(freqs, dtype=torch.float64)[:, None]
        c = SpectralDescriptors.spectral_centroid(m, freqs)
        w = m / m.sum(-2, keepdim=True).clamp_min(1e-300)
        return ((w * (f - c.unsqueeze(-2)).abs() ** p).sum(-2)) ** (1.0 / p)

    @staticmethod
    def spectral_rolloff(mag, freqs, roll_percent: float = 0.85) -> torch.Tensor:
        """Lowest bin frequency below which roll_percent of the frame's magnitude lies."""
        m = mag.double()
        cum = m.cumsum(-2)
        thr = roll_percent * cum[..., -1:, :]
        idx = (cum < thr).sum(-2).clamp(max=m.shape[-2] - 1)
        return torch.as_tensor(freqs, dtype=torch.float64)[idx]

    @staticmethod
    def spectral_flatness(mag, eps: float = 1e-10) -> torch.Tensor:
        """Geometric over arithmetic mean of the power spectrum (1 for white noise, near 0 for a tone)."""
        p = mag.double() ** 2 + eps
        return torch.exp(torch.log(p).mean(-2)) / p.mean(-2)


def spectral_flux(mag: torch.Tensor) -> torch.Tensor:
    """L2 norm of the positive magnitude change between consecutive frames (0 for the first frame)."""
    m = mag.double()
    d = (m[..., 1:] - m[..., :-1]).clamp_min(0)
    return torch.cat([torch.zeros(*m.shape[:-2], 1, dtype=m.dtype), d.square().sum(-2).sqrt()], -1)


def zero_crossing_rate(signal: torch.Tensor, frame_size: int, hop_size: int) -> torch.Tensor:
    """Fraction of adjacent sample pairs with a sign change, per frame."""
    x = torch.as_tensor(signal, dtype=torch.float64)
    if x.shape[-1] < frame_size:
        return x.new_zeros(*x.shape[:-1], 0)
    f = x.unfold(-1, frame_size, hop_size)
    s = torch.sign(f)
    return (s[..., 1:] * s[..., :-1] < 0).double().sum(-1) / max(frame_size - 1, 1)


def chroma_cens(chroma: torch.Tensor, window_size: int = 41) -> torch.Tensor:
    """Chroma energy normalised statistics (Mueller et al. 2005) from a [12, frames] chromagram: L1-normalise
    each frame, quantise into 5 logarithmic levels (thresholds 0.05, 0.1, 0.2, 0.4), smooth over time with a
    Hann window and L2-normalise each frame."""
    c = torch.as_tensor(chroma, dtype=torch.float64)
    c = c / c.abs().sum(-2, keepdim=True).clamp_min(1e-12)
    q = sum((c > t).double() for t in (0.05, 0.1, 0.2, 0.4))
    w = torch.hann_window(window_size + 2, periodic=False, dtype=torch.float64)[1:-1]
    w = w / w.sum()
    pad = window_size // 2
    qp = torch.nn.functional.pad(q.reshape(-1, 1, q.shape[-1]), (pad, window_size - 1 - pad))
    sm = torch.nn.functional.conv1d(qp, w.view(1, 1, -1)).reshape(q.shape)
    return sm / sm.norm(dim=-2, keepdim=True).clamp_min(1e-12)
