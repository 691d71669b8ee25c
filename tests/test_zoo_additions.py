"""SAC, world model and curiosity (crates/brain-rl), spectral denoising (crates/brain-audio/src/denoise.rs)
and fastText subword embeddings (crates/brain-text/src/embedding/fasttext.rs)."""
import math

import torch

from brain_b200 import text
from brain_b200.zoo import audio, rl


def test_world_model_matches_reference_construction_and_trains():
    wm = rl.WorldModel(4, 2, 16)
    scale = math.sqrt(2.0 / 6)
    assert abs(float(wm.w_embed[0, 1]) - math.sin(0.1337) * scale) < 1e-6
    assert abs(float(wm.w_state[0, 1]) - math.cos(0.7331) * scale) < 1e-6
    s = torch.tensor([1.0, 0.5, -0.2, 0.8])
    a = torch.tensor([0.1, -0.5])
    nxt, r = wm.predict(s, a)
    assert nxt.shape == (4,) and float(wm.loss(s, a, nxt, r)) < 1e-6  # the reference test
    # learn a linear dynamics model from samples
    torch.manual_seed(0)
    S, A = torch.randn(256, 4), torch.randn(256, 2)
    S2, R = S + 0.1 * A.repeat(1, 2), A.sum(-1)
    opt = torch.optim.Adam(wm.parameters(), lr=1e-2)
    first = float(wm.loss(S, A, S2, R))
    for _ in range(200):
        loss = wm.loss(S, A, S2, R)
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert float(loss) < 0.1 * first


def test_curiosity_reward_and_training():
    icm = rl.IntrinsicCuriosityModule(4, 2, 8, 0.1)
    s, a = torch.tensor([1.0, 0.5, -0.2, 0.8]), torch.tensor([0.1, -0.5])
    s2 = torch.tensor([1.1, 0.4, -0.1, 0.7])
    r = icm.compute_intrinsic_reward(s, a, s2)
    assert float(r) >= 0.0
    phi = icm.encode_state(s)
    w = math.sqrt(2.0 / 4)
    manual = sum(math.sin(0.177 * j) * w * float(s[j]) for j in range(4))
    assert abs(float(phi[0]) - (manual if manual >= 0 else 0.01 * manual)) < 1e-5
    torch.manual_seed(1)
    S, A = torch.randn(128, 4), torch.randn(128, 2)
    S2 = S + 0.2 * torch.cat([A, A], -1)
    opt = torch.optim.Adam(icm.parameters(), lr=1e-2)
    first = float(icm.loss(S, A, S2))
    for _ in range(150):
        loss = icm.loss(S, A, S2)
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert float(loss) < 0.5 * first


def test_sac_learns_a_one_step_task():
    """Reward -||a - target(s)||^2 for a 1-D target: SAC's deterministic action approaches it."""
    torch.manual_seed(0)
    agent = rl.SacAgent(2, 1, rl.SacConfig(lr=3e-3, hidden=32, target_entropy=-1.0), seed=0)
    assert abs(rl.SacAgent(2, 1).alpha() - 0.2) < 1e-6
    for it in range(400):
        s = torch.randn(64, 2)
        a = torch.tanh(torch.randn(64, 1))
        r = -((a - 0.5 * torch.tanh(s[:, :1])) ** 2).sum(-1)
        info = agent.update(s, a, r, s, torch.ones(64))
    s = torch.randn(256, 2)
    err = ((torch.stack([agent.act(x, deterministic=True) for x in s]) - 0.5 * torch.tanh(s[:, :1])) ** 2).mean()
    assert float(err) < 0.05, float(err)
    assert set(info) == {"q_loss", "actor_loss", "alpha_loss", "alpha"}


def test_spectral_denoising_improves_snr():
    torch.manual_seed(0)
    sr, n = 16000, 16000
    t = torch.arange(n) / sr
    clean = 0.5 * torch.sin(2 * math.pi * 440 * t)
    clean[:2000] = 0.0  # leading noise-only frames for the noise estimate
    noisy = clean + 0.05 * torch.randn(n)
    before = audio.snr_db(clean, noisy)
    ss = audio.spectral_subtraction(noisy, oversubtraction=2.0, spectral_floor=0.01)
    wf = audio.wiener_filter(noisy)
    assert ss.shape == noisy.shape and wf.shape == noisy.shape
    assert audio.snr_db(clean, ss) > before + 3.0
    assert audio.snr_db(clean, wf) > before + 3.0
    # minimum statistics tracks the floor between bursts (a stationary tone would be taken for noise)
    bursts = clean * ((t * 2).floor() % 2 == 0).float()
    noisy_b = bursts + 0.05 * torch.randn(n)
    wf_ms = audio.wiener_filter(noisy_b, min_stats=True)
    assert audio.snr_db(bursts, wf_ms) > audio.snr_db(bursts, noisy_b)
    mag, _ = audio.stft(noisy)
    floor = audio.minimum_statistics_noise(mag ** 2)
    assert floor.shape == mag.shape and bool((floor <= (mag ** 2).max()).all())


def test_fasttext_subwords_and_oov():
    cfg = text.FastTextConfig(dim=8, bucket_size=100, min_n=3, max_n=4)
    ft = text.FastTextEmbedding(cfg)
    assert ft.extract_subwords("ab") == ["<ab", "ab>", "<ab>"]
    assert text.FastTextEmbedding.compute_ngram_hash("", 1 << 62) == 0xCBF29CE484222325 % (1 << 62)
    ft.insert_word("apple", [0.1] * 8)
    ft.insert_word("application_1", [0.2] * 8)
    assert ft.get_word_vector("apple").shape == (8,)
    assert float(ft.get_word_vector("applesauce").abs().sum()) > 0  # OOV word shares n-grams with apple
    big = text.FastTextEmbedding(text.FastTextConfig(dim=8, bucket_size=1 << 20, min_n=3, max_n=4))
    big.insert_word("apple", [0.1] * 8)
    assert float(big.get_word_vector("zzzz").abs().sum()) == 0.0  # no shared n-gram, no collision
    sim = ft.most_similar("apples", ["apple", "banana", "car"], 2)
    assert len(sim) == 2 and sim[0][0] == "apple"
    batch = ft.word_vectors(["apple", "applesauce", "zzzz"])
    torch.testing.assert_close(batch[0], ft.get_word_vector("apple"))
    torch.testing.assert_close(batch[1], ft.get_word_vector("applesauce"))
