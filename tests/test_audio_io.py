"""Audio buffers, FLAC / MPEG header parsing, mel and Bark scales, deltas, spectral descriptors, zero-crossing
rate and CENS chroma (crates/brain-audio/src/core.rs, io/flac.rs, io/mp3.rs, utils.rs, feature/spectral.rs,
feature/tonal.rs)."""
import math

import pytest
import torch

from brain_b200.zoo import audio_io as AI


def test_audio_buffer_ops():
    b = AI.AudioBuffer(torch.tensor([[1.0, -2.0, 3.0], [3.0, 2.0, 1.0]]), 8000)
    assert b.channels == 2 and b.num_samples == 3 and b.duration() == pytest.approx(3 / 8000)
    assert b.to_mono().data.tolist() == [[2.0, 0.0, 2.0]]
    assert b.slice(1, 3).data.tolist() == [[-2.0, 3.0], [2.0, 1.0]]
    m = AI.AudioBuffer(torch.tensor([0.5, -0.25]), 8000)
    assert m.to_stereo().channels == 2 and m.concat(m).num_samples == 4
    b2 = b.slice(0, 3)
    b2.mix(b, 0.5)
    assert b2.data[0].tolist() == [1.5, -3.0, 4.5]
    b2.normalize_peak(1.0)
    assert b2.peak_amplitude() == pytest.approx(1.0)
    with pytest.raises(ValueError):
        b.concat(m)


def test_flac_and_mpeg_headers():
    info = bytearray(b"fLaC")
    info += bytes([0x80, 0, 0, 34])  # last-block flag + STREAMINFO, length 34
    info += (4096).to_bytes(2, "big") + (4096).to_bytes(2, "big") + (14).to_bytes(3, "big") + (9000).to_bytes(3, "big")
    word = (44100 << 44) | ((2 - 1) << 41) | ((16 - 1) << 36) | 1234567
    info += word.to_bytes(8, "big") + bytes(16)
    si = AI.parse_flac_metadata(bytes(info))
    assert (si.sample_rate, si.channels, si.bits_per_sample, si.total_samples) == (44100, 2, 16, 1234567)
    assert (si.min_block_size, si.max_frame_size) == (4096, 9000)
    with pytest.raises(ValueError):
        AI.parse_flac_metadata(b"OggS" + bytes(40))
    # MPEG-1 layer III, 128 kbit/s, 44.1 kHz, no padding, joint stereo
    h = bytes([0xFF, 0xFB, 0x90, 0x40])
    hdr = AI.Mp3FrameHeader.parse(h)
    assert (hdr.version, hdr.layer, hdr.bitrate_kbps, hdr.sample_rate, hdr.channels) == (1, 3, 128, 44100, 2)
    assert hdr.frame_size == 144 * 128000 // 44100
    # MPEG-2 layer III, 64 kbit/s (index 8), 22.05 kHz, padded, mono
    h2 = bytes([0xFF, 0xF3, 0x82, 0xC0])
    hdr2 = AI.Mp3FrameHeader.parse(h2)
    assert (hdr2.version, hdr2.bitrate_kbps, hdr2.sample_rate, hdr2.channels) == (2, 64, 22050, 1)
    assert hdr2.frame_size == 72 * 64000 // 22050 + 1
    stream = b"\x00\x01" + (h + bytes(hdr.frame_size - 4)) * 3 + b"\xff"
    assert len(AI.parse_mp3_frames(stream)) == 3


def test_scales_deltas_descriptors():
    for f in (100.0, 700.0, 1000.0, 4000.0):
        assert float(AI.mel_to_hz_htk(AI.hz_to_mel_htk(f))) == pytest.approx(f)
        assert float(AI.mel_to_hz_slaney(AI.hz_to_mel_slaney(f))) == pytest.approx(f)
        assert float(AI.bark_to_hz(AI.hz_to_bark(f))) == pytest.approx(f)
    assert float(AI.hz_to_mel_slaney(1000.0)) == pytest.approx(15.0)
    x = torch.arange(10, dtype=torch.float64).repeat(2, 1)
    d = AI.compute_deltas(x, 1, 5)
    assert d[0, 5] == pytest.approx(1.0) and d[0, 0] == pytest.approx((1 * 1 + 2 * 2) / 10)
    assert torch.allclose(AI.compute_deltas(x, 2, 5)[:, 4:6], torch.zeros(2, 2, dtype=torch.float64))  # away from the edges
    mag = torch.zeros(5, 3, dtype=torch.float64)
    mag[1, 0] = 1.0
    mag[3, 1] = 2.0
    mag[:, 2] = 1.0
    freqs = torch.tensor([0.0, 100.0, 200.0, 300.0, 400.0])
    assert AI.SpectralDescriptors.spectral_centroid(mag, freqs).tolist() == pytest.approx([100.0, 300.0, 200.0])
    assert AI.SpectralDescriptors.spectral_rolloff(mag, freqs, 0.85).tolist() == [100.0, 300.0, 400.0]
    assert float(AI.SpectralDescriptors.spectral_bandwidth(mag, freqs)[0]) == pytest.approx(0.0)
    fl = AI.SpectralDescriptors.spectral_flatness(mag)
    assert float(fl[2]) == pytest.approx(1.0) and float(fl[0]) < 0.01
    fx = AI.spectral_flux(mag)
    assert fx[0] == 0.0 and float(fx[1]) == pytest.approx(2.0)
    z = AI.zero_crossing_rate(torch.tensor([1.0, -1.0, 1.0, -1.0, 1.0, 1.0]), 3, 3)
    assert z.tolist() == [1.0, 0.5]
    ch = torch.rand(12, 50, dtype=torch.float64)
    cens = AI.chroma_cens(ch, 9)
    assert cens.shape == (12, 50) and torch.allclose(cens.norm(dim=0), torch.ones(50, dtype=torch.float64))
