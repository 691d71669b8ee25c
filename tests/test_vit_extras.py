"""ViT utilities against restatements of crates/brain-vit/src (patch/pos_embed.rs, utils.rs, ops.rs,
vit/heads.rs, export/mod.rs)."""
import math

import pytest
import torch

from brain_b200.models import vit_extras as VX


def test_sinusoidal_tables():
    t = VX.sinusoidal_1d(5, 6)
    assert float(t[3, 2]) == pytest.approx(math.sin(3 / 10000 ** (2 * 1 / 6)))
    assert float(t[3, 3]) == pytest.approx(math.cos(3 / 10000 ** (2 * 1 / 6)))
    t2 = VX.sinusoidal_2d(3, 4, 8)
    h, w, i = 2, 3, 1
    om = 1 / 10000 ** (2 * i / 8)
    assert float(t2[h * 4 + w, 2 * i]) == pytest.approx(math.sin(h * om))
    assert float(t2[h * 4 + w, 2 * i + 1]) == pytest.approx(math.cos(w * om))


def test_interpolation_and_pos_embed_resize():
    g = torch.arange(6, dtype=torch.float64).view(2, 3)
    out = VX.interpolate_2d(g, 3, 5)
    assert out[0, 0] == 0 and out[-1, -1] == 5 and float(out[1, 2]) == pytest.approx(2.5)
    torch.testing.assert_close(VX.interpolate_2d(g, 2, 3), g)
    pos = torch.randn(1, 1 + 4 * 4, 8, dtype=torch.float64)
    new = VX.interpolate_pos_embed(pos, (4, 4), (6, 6))
    assert new.shape == (1, 1 + 36, 8) and torch.equal(new[:, 0], pos[:, 0])
    torch.testing.assert_close(new[0, 1].double(), pos[0, 1])  # corners are kept
    torch.testing.assert_close(new[0, -1], pos[0, -1])


def test_patch_token_ops():
    img = torch.randn(2, 3, 8, 12)
    tok = VX.patchify(img, 4)
    assert tok.shape == (2, 6, 48)
    torch.testing.assert_close(tok[1, 4].view(3, 4, 4), img[1, :, 4:8, 4:8])
    torch.testing.assert_close(VX.unpatchify(tok, 4, 3, 8, 12), img)
    cls = torch.ones(48)
    t2 = VX.add_cls_token(tok, cls)
    c, rest = VX.split_cls_token(t2)
    assert torch.equal(rest, tok) and float(c.sum()) == 2 * 48
    keep = torch.tensor([True, False, True, False, False, True])
    kept, idx = VX.mask_patches(tok, keep)
    assert idx.tolist() == [0, 2, 5] and torch.equal(kept[:, 1], tok[:, 2])
    m = VX.random_keep_mask(16, 0.75, torch.Generator().manual_seed(0))
    assert int(m.sum()) == 4
    s = VX.stochastic_depth_scale(0.5, True, 1000, torch.Generator().manual_seed(1))
    assert set(s.tolist()) <= {0.0, 2.0} and abs(float(s.mean()) - 1.0) < 0.15
    assert torch.equal(VX.stochastic_depth_scale(0.5, False, 3), torch.ones(3))


def test_rollout_entropy_ntxent_dino_card():
    a = torch.softmax(torch.randn(3, 5, 5, dtype=torch.float64), -1)
    r = VX.attention_rollout(a)
    ref = torch.eye(5, dtype=torch.float64)
    for l in range(3):
        ref = (0.5 * a[l] + 0.5 * torch.eye(5, dtype=torch.float64)) @ ref
    torch.testing.assert_close(r, ref)
    torch.testing.assert_close(r.sum(-1), torch.ones(5, dtype=torch.float64))  # rows stay stochastic
    u = torch.full((2, 4), 0.25, dtype=torch.float64)
    assert VX.attention_entropy(u).tolist() == pytest.approx([math.log(4)] * 2)
    z1, z2 = torch.randn(3, 4, dtype=torch.float64), torch.randn(3, 4, dtype=torch.float64)
    z = torch.cat([z1, z2])
    sim = z @ z.t() / 0.5
    want = 0.0
    for i in range(6):
        j = (i + 3) % 6
        others = [sim[i, k] for k in range(6) if k != i]
        want += float(torch.logsumexp(torch.stack(others), 0) - sim[i, j])
    assert float(VX.nt_xent_loss(z1, z2, 0.5)) == pytest.approx(want / 6)
    head = VX.DinoHead(8, 16, 4)
    out = head(torch.randn(5, 8))
    torch.testing.assert_close(out.norm(dim=-1), torch.ones(5))
    with pytest.raises(ValueError):
        VX.DinoHead(0, 4, 4)
    card = VX.ModelCard.for_model("vit-tiny", head, {"patch": 16})
    card.add_metric("top1", 0.5)
    md = card.to_markdown()
    assert "# vit-tiny" in md and "| top1 | 0.5000 |" in md and "patch: 16" in md
