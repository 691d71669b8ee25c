"""GAN losses, regularisers, StyleGAN/CycleGAN pieces, evaluation metrics and sampling utilities against
restatements of crates/brain-gan/src (losses/classic.rs, losses/perceptual.rs, cycle.rs, ops.rs,
stylegan_lite.rs, utils.rs, eval/, train/penalties.rs)."""
import math

import pytest
import torch

from brain_b200.zoo import gan_extras as GE

M64 = (1 << 64) - 1


def test_relativistic_and_perceptual_losses():
    assert float(GE.ragan_loss_d(torch.tensor(2.0), torch.tensor(0.5))) == pytest.approx(max(0, 1 - 1.5) + max(0, 1 - 1.5))
    assert float(GE.ragan_loss_g(torch.tensor(0.2), torch.tensor(0.7))) == pytest.approx(max(0, 1 - 0.5) + max(0, 1 - 0.5))
    v = torch.tensor([1.0, 2.0, 3.0])
    assert GE.gram_matrix(v).tolist() == [[1, 2, 3], [2, 4, 6], [3, 6, 9]]
    f = torch.randn(2, 3, 4, 4)
    g = GE.gram_matrix(f)
    torch.testing.assert_close(g[1, 0, 2], (f[1, 0] * f[1, 2]).sum())
    assert float(GE.feature_matching_loss(torch.tensor([1.0, 2.0, 3.0]), torch.tensor([1.0, 0.0]))) == pytest.approx(2.0)
    r, q = torch.randn(6), torch.randn(6)
    want = 10.0 * float(((r - q) ** 2).mean()) + float(((torch.outer(r, r) - torch.outer(q, q)) ** 2).mean())
    assert float(GE.perceptual_loss(r, q)) == pytest.approx(want, rel=1e-5)
    assert float(GE.cycle_consistency_loss(torch.tensor([1.0, -1.0]), torch.tensor([0.0, 1.0]))) == 1.5
    assert GE.cycle_total_loss(1.0, 2.0, 3.0) == 1.0 + 20.0 + 15.0


def test_spectral_norm_power_iteration_converges():
    torch.manual_seed(0)
    w = torch.randn(8, 5, dtype=torch.float64)
    u = torch.randn(8, dtype=torch.float64)
    for _ in range(50):
        w_sn, u, sigma = GE.spectral_norm_apply(w, u)
    assert sigma == pytest.approx(float(torch.linalg.matrix_norm(w, 2)), rel=1e-6)
    assert float(torch.linalg.matrix_norm(w_sn, 2)) == pytest.approx(1.0, rel=1e-6)


def test_latents_grid_adain_style_mix_ema():
    a, b = torch.zeros(4), torch.ones(4)
    assert GE.interpolate_latents(a, b, 0.25).tolist() == [0.75] * 4
    seq = GE.interpolate_latents_batch(a, b, 4)
    assert seq.shape == (5, 4) and seq[0].tolist() == [1.0] * 4 and seq[4].tolist() == [0.0] * 4
    imgs = torch.arange(5 * 3 * 2 * 2, dtype=torch.float32).view(5, 3, 2, 2)
    grid = GE.image_grid(imgs, 3, pad=1)
    assert grid.shape == (3, 2 * 3 - 1, 3 * 3 - 1)
    torch.testing.assert_close(grid[:, 3:5, 3:5], imgs[4])
    x = torch.randn(2, 3, 5, 5)
    sc, bi = torch.rand(2, 3) + 0.5, torch.randn(2, 3)
    y = GE.adaptive_instance_norm(x, sc, bi)
    torch.testing.assert_close(y.mean((2, 3)), bi, atol=1e-5, rtol=0)
    torch.testing.assert_close(y.std((2, 3), unbiased=False), sc, atol=1e-3, rtol=1e-3)
    ws = GE.style_mix(a, b, 2, 5)
    assert [bool(t.sum() == 0) for t in ws] == [True, True, False, False, False]
    ema = [torch.zeros(3)]
    GE.track_ema(ema, [torch.ones(3)], 0.9)
    assert ema[0].tolist() == pytest.approx([0.1] * 3)
    assert GE.smooth_labels(1.0) == (0.9, 0.0) and GE.clip_weights(torch.tensor([2.0, -3.0]), 1.0).tolist() == [1.0, -1.0]


def test_lcg_sampling_and_eval_metrics():
    z = GE.sample_gaussian(3, 7)
    s, ref = 7, []
    for _ in range(3):
        s = (s * 6364136223846793005 + 1442695040888963407) & M64
        u1 = max((s >> 11) / float(1 << 53), 1e-15)
        s = (s * 6364136223846793005 + 1442695040888963407) & M64
        u2 = (s >> 11) / float(1 << 53)
        ref.append(math.sqrt(-2 * math.log(u1)) * math.cos(2 * math.pi * u2))
    assert z.tolist() == pytest.approx(ref)
    fl = GE.fixed_latent_sample(3, 2, 7)
    assert fl[0].tolist() == pytest.approx(ref) and fl.shape == (2, 3)
    real, fake = torch.ones(4, 3), torch.zeros(4, 3)
    assert GE.fid_lite(real, fake) == 3.0
    assert GE.is_lite(torch.zeros(5, 10)) == pytest.approx(math.e)  # uniform: entropy = ln(10)
    rep = GE.eval_gan(real, fake)
    assert rep.num_samples == 4 and rep.avg_d_real == pytest.approx(math.tanh(3.0)) and "FID-lite" in rep.summary()


def test_stylegan_and_cyclegan_modules_train():
    torch.manual_seed(0)
    sg = GE.StyleGanLite(latent_dim=16, style_dim=16, output_size=16, channels=8, mapping_layers=2)
    img = sg(torch.randn(3, 16))
    assert img.shape == (3, 3, 16, 16) and float(img.detach().abs().max()) <= 1.0
    w1, w2 = sg.mapping(torch.randn(3, 16)), sg.mapping(torch.randn(3, 16))
    mixed = sg.synthesize(GE.style_mix(w1, w2, 2, sg.num_layers))
    assert mixed.shape == img.shape
    cg = GE.CycleGan(6, 32)
    opt = torch.optim.Adam(cg.parameters(), lr=1e-2)
    a, b = torch.rand(16, 6) * 0.5, torch.rand(16, 6) * 0.5
    first = None
    for _ in range(30):
        loss, *_ = cg.generator_losses(a, b)
        first = first if first is not None else float(loss.detach())
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert float(loss) < first


def test_patch_resnet_conditional_and_trainer():
    import torch
    from brain_b200.zoo import gan_extras as GX
    from brain_b200.zoo.gan import MlpDiscriminator, MlpGenerator
    torch.manual_seed(0)
    pd = GX.PatchDiscriminator(3, base=8, n_layers=3)
    out = pd(torch.randn(2, 3, 64, 64))
    assert out.shape == (2, 1, 8, 8) and pd.num_patches(64, 64) == 64
    rg = GX.ResnetGenerator(3, 3, base=8, n_blocks=2, norm="instance")
    y = rg(torch.randn(1, 3, 32, 32))
    assert y.shape == (1, 3, 32, 32) and y.abs().max() <= 1
    cg = GX.ConditionalGenerator(8, 4, 10, hidden=16)
    cd = GX.ConditionalDiscriminator(10, 4, hidden=16)
    z = torch.randn(5, 8)
    labels = torch.tensor([0, 1, 2, 3, 0])
    x = cg(z, labels)
    assert x.shape == (5, 10)
    assert not torch.allclose(cg(z, torch.zeros(5, dtype=torch.long)), cg(z, torch.ones(5, dtype=torch.long)))
    s = cd(x, labels)
    h = cd.phi(x)
    assert torch.allclose(s, cd.out(h) + (cd.class_embed(labels) * h).sum(-1, keepdim=True))
    gen = MlpGenerator(4, 2, hidden=16)
    disc = MlpDiscriminator(2, hidden=16)
    tr = GX.GanTrainer(gen, disc, torch.optim.Adam(gen.parameters(), 1e-3), torch.optim.Adam(disc.parameters(), 1e-3),
                       loss="wgan", n_critic=2, clip=0.05)
    data = lambda: [torch.randn(16, 2) * 0.1 + 1.0 for _ in range(4)]
    hist = tr.fit(data, 2)
    assert len(hist) == 2 and hist[1].steps == 4 and all(p.abs().max() <= 0.05 + 1e-7 for p in disc.parameters())
    g = GX.assemble_grid(torch.zeros(3, 1, 4, 4), 2, pad=1)
    assert g.shape == (1, 9, 9)
