"""Audio helpers: dB conversions, windows, ERB scale, Hilbert envelope, cepstrum, phase vocoder."""
import math

import pytest
import torch

from brain_b200.zoo import audio_fx as A


def test_db_windows_scales():
    x = torch.tensor([1.0, 10.0, 100.0])
    assert torch.allclose(A.amplitude_to_db(x), torch.tensor([0.0, 20.0, 40.0]))
    assert torch.allclose(A.power_to_db(x), torch.tensor([0.0, 10.0, 20.0]))
    assert torch.allclose(A.db_to_amplitude(A.amplitude_to_db(x)), x) and torch.allclose(A.db_to_power(A.power_to_db(x)), x)
    assert torch.allclose(A.power_to_db(x, top_db=5.0), torch.tensor([15.0, 15.0, 20.0]))
    assert A.bartlett_window(8).shape == (8,) and float(A.blackman_window(9, periodic=False)[4]) == pytest.approx(1.0)
    assert float(A.erb_to_hz(A.hz_to_erb(1000.0))) == pytest.approx(1000.0)
    assert float(A.hz_to_erb(1000.0)) == pytest.approx(21.4 * math.log10(1 + 4.37), rel=1e-9)
    assert A.samples_from_duration(0.5, 16000) == 8000 and A.nyquist_hz(16000) == 8000.0
    assert A.fft_freqs(8, 16).tolist() == [0.0, 2.0, 4.0, 6.0, 8.0]
    assert A.ensure_length(torch.ones(3), 5).tolist() == [1, 1, 1, 0, 0] and A.ensure_length(torch.ones(6), 2).shape == (2,)
    assert A.vector_distance(torch.tensor([3.0, 0]), torch.tensor([0.0, 4])) == 5.0
    assert A.vector_distance(torch.tensor([1.0, 0]), torch.tensor([2.0, 0]), "cosine") == pytest.approx(0.0)
    sp, mu = A.MelConfig.default_speech(), A.MelConfig.default_music_128()
    assert (sp.n_mels, mu.n_mels, mu.sample_rate) == (80, 128, 22050)


def test_envelope_cepstrum_deemphasis_vocoder():
    sr = 8000
    t = torch.arange(4000, dtype=torch.float64) / sr
    env = 1.0 + 0.5 * torch.sin(2 * math.pi * 3 * t)
    x = env * torch.sin(2 * math.pi * 1000 * t)
    e = A.hilbert_envelope(x)
    assert float((e[200:-200] - env[200:-200]).abs().max()) < 0.02
    c = A.real_cepstrum(torch.randn(256, dtype=torch.float64))
    assert c.shape == (256,) and torch.isfinite(c).all()
    y = torch.randn(50, dtype=torch.float64)
    pre = torch.cat([y[:1], y[1:] - 0.97 * y[:-1]])
    assert torch.allclose(A.de_emphasis(pre, 0.97), y)
    tone = torch.sin(2 * math.pi * 440 * torch.arange(16000) / 16000).float()
    pv = A.PhaseVocoder(1024, 256)
    slow = pv.stretch(tone, 0.5)
    assert abs(slow.shape[-1] - 32000) <= 1
    spec = torch.fft.rfft(slow[4000:28000].double()).abs()
    peak = int(spec.argmax()) * 16000 / 24000
    assert abs(peak - 440) < 5  # the pitch is kept while the duration doubles
