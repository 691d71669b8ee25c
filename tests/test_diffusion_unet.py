"""Diffusion U-Net, PLMS sampling, guidance, conditioning and training (crates/brain-diffusion/src/unet,
samplers/plms.rs, guidance.rs, conditioning.rs, diffusion/train.rs)."""
import torch

from brain_b200.zoo.diffusion import DdimSampler, LinearSchedule
from brain_b200.zoo import diffusion_unet as DU


def _sched():
    return LinearSchedule(200)


def test_unet_shapes_with_and_without_cross_attention():
    torch.manual_seed(0)
    cfg = DU.UnetConfig(in_channels=3, out_channels=3, model_channels=16, num_res_blocks=1, channel_mult=(1, 2),
                        attention_levels=(1,), num_heads=2, context_dim=8, groups=8)
    net = DU.Unet2d(cfg)
    x = torch.randn(2, 3, 16, 16)
    out = net(x, torch.tensor([3, 7]), torch.randn(2, 5, 8))
    assert out.shape == x.shape
    assert net(x, 5).shape == x.shape  # scalar timestep, no context
    loss = out.square().mean()
    loss.backward()
    assert all(p.grad is not None for p in net.parameters() if p.requires_grad and p.dim() > 1)


def test_plms_and_ddim_recover_x0_with_an_oracle_denoiser():
    s = _sched()
    x0 = torch.randn(3, 4, dtype=torch.float64)

    def oracle(x, t, cond=None):
        ac = s.alphas_cumprod[t].view(-1, 1).to(x.dtype)
        return (x - ac.sqrt() * x0) / (1 - ac).sqrt()

    for sampler in (DU.PlmsSampler(s), DdimSampler(s)):
        out = sampler.sample(oracle, (3, 4), num_steps=20, generator=torch.Generator().manual_seed(1),
                             dtype=torch.float64)
        torch.testing.assert_close(out, x0, rtol=1e-6, atol=1e-6)


def test_cfg_context_codec_and_trainer():
    u, c = torch.zeros(2), torch.ones(2)
    assert DU.apply_cfg(u, c, 3.0).tolist() == [3.0, 3.0]
    ctx = DU.ConditioningContext(torch.ones(6, 2, 3))
    dropped = ctx.drop(1.0)
    assert float(dropped.abs().sum()) == 0.0 and torch.equal(ctx.drop(0.0), ctx.context)
    codec = DU.IdentityLatentCodec()
    z = torch.randn(2, 2)
    assert torch.equal(codec.decode(codec.encode(z)), z)
    torch.manual_seed(0)
    cfg = DU.UnetConfig(in_channels=1, out_channels=1, model_channels=8, num_res_blocks=1, channel_mult=(1, 2),
                        attention_levels=(), num_heads=2, groups=4)
    net = DU.Unet2d(cfg)
    tr = DU.DiffusionTrainer(net, _sched(), lr=3e-3, ema_decay=0.9)
    data = torch.zeros(8, 1, 8, 8)
    data[:, :, 2:6, 2:6] = 1.0
    g = torch.Generator().manual_seed(0)
    losses = [tr.step(data, generator=g) for _ in range(40)]
    assert sum(losses[-5:]) / 5 < sum(losses[:5]) / 5
    assert tr.steps == 40 and len(tr.ema) == len(list(net.parameters()))
