"""CV operators and blocks against direct restatements (crates/brain-cv/src/ops, augmentation, detection/roi.rs,
conv/deformable.rs, conv/residual.rs, feature/backbones.rs)."""
import colorsys
import math

import pytest
import torch
import torch.nn.functional as F

from brain_b200.zoo import cv_extras as CX


def test_box_ops_and_formats():
    a = torch.tensor([[0.0, 0.0, 2.0, 2.0], [1.0, 1.0, 3.0, 4.0]], dtype=torch.float64)
    b = torch.tensor([[1.0, 1.0, 2.0, 2.0], [5.0, 5.0, 6.0, 6.0]], dtype=torch.float64)
    assert CX.box_area(a).tolist() == [4.0, 6.0]
    iou = CX.box_iou_matrix(a, b)
    assert float(iou[0, 0]) == pytest.approx(1 / 4) and float(iou[0, 1]) == 0.0
    giou = CX.box_giou_matrix(a, b)
    enc = 36.0  # (0,0)-(6,6)
    assert float(giou[0, 1]) == pytest.approx(0.0 - (enc - 5.0) / enc)
    for f in ("xywh", "cxcywh"):
        torch.testing.assert_close(CX.convert_bbox_format(CX.convert_bbox_format(a, "xyxy", f), f, "xyxy"), a)
    assert CX.convert_bbox_format(a, "xyxy", "cxcywh")[1].tolist() == [2.0, 2.5, 2.0, 3.0]
    assert CX.transform_bounding_boxes(a, 10.0, True)[0].tolist() == [8.0, 0.0, 10.0, 2.0]


def test_photometric_and_color_spaces():
    img = torch.rand(2, 3, 8, 8, dtype=torch.float64)
    s = CX.solarize(img, 0.5)
    assert torch.equal(s[img < 0.5], img[img < 0.5]) and torch.allclose(s[img >= 0.5], 1 - img[img >= 0.5])
    eq = CX.equalize((img * 0.3 + 0.2).float())
    assert float(eq.min()) == 0.0 and float(eq.max()) == pytest.approx(1.0)
    hsv = CX.rgb_to_hsv(img)
    px = img[0, :, 3, 5].tolist()
    want = colorsys.rgb_to_hsv(*px)
    assert hsv[0, :, 3, 5].tolist() == pytest.approx(list(want))
    torch.testing.assert_close(CX.hsv_to_rgb(hsv), img)
    torch.testing.assert_close(CX.yuv_to_rgb(CX.rgb_to_yuv(img)), img)
    lab = CX.rgb_to_lab(torch.ones(1, 3, 1, 1, dtype=torch.float64))
    assert lab.view(-1).tolist() == pytest.approx([100.0, 0.0, 0.0], abs=1e-3)  # white
    assert CX.convert_color(img, "rgb", "grayscale").shape == (2, 1, 8, 8)
    cj = CX.ColorJitter(0.3, 0.3, 0.3, 0.1, generator=torch.Generator().manual_seed(0))
    out = cj(img.float())
    assert out.shape == img.shape and float(out.min()) >= -1e-6 and float(out.max()) <= 1 + 1e-6


def test_geometry_crop_compose():
    theta = torch.tensor([[[1.0, 0.0, 0.0], [0.0, 1.0, 0.0]]])
    x = torch.rand(1, 2, 5, 7)
    grid = CX.affine_grid(theta, (1, 2, 5, 7), align_corners=True)
    torch.testing.assert_close(CX.grid_sample(x, grid, align_corners=True), x)
    rrc = CX.RandomResizedCrop(4, seed=1)
    assert rrc(torch.rand(3, 20, 30)).shape == (3, 4, 4)
    comp = CX.Compose([lambda t: t + 1, lambda t: t * 2])
    assert comp(torch.ones(1)).tolist() == [4.0]


def test_roi_pool_matches_loop():
    torch.manual_seed(0)
    feat = torch.randn(2, 3, 10, 12)
    rois = torch.tensor([[0, 1.0, 2.0, 9.0, 7.0], [1, 0.0, 0.0, 11.0, 9.0], [1, 4.0, 4.0, 4.0, 4.0]])
    out = CX.RoIPool((2, 3), 1.0)(feat, rois)
    assert out.shape == (3, 3, 2, 3)
    for r in range(3):
        b, x1, y1, x2, y2 = [int(round(v)) for v in rois[r].tolist()]
        rw, rh = max(x2 - x1 + 1, 1), max(y2 - y1 + 1, 1)
        for i in range(2):
            hs, he = min(max(y1 + math.floor(i * rh / 2), 0), 10), min(max(y1 + math.ceil((i + 1) * rh / 2), 0), 10)
            for j in range(3):
                ws, we = min(max(x1 + math.floor(j * rw / 3), 0), 12), min(max(x1 + math.ceil((j + 1) * rw / 3), 0), 12)
                if he > hs and we > ws:
                    torch.testing.assert_close(out[r, :, i, j], feat[b, :, hs:he, ws:we].amax((1, 2)))


def test_deformable_conv_zero_offsets_equals_conv():
    torch.manual_seed(0)
    dc = CX.DeformableConv2d(3, 4, 3, stride=1, padding=1)
    x = torch.randn(2, 3, 6, 7)
    off = torch.zeros(2, 18, 6, 7)
    torch.testing.assert_close(dc(x, off), F.conv2d(x, dc.weight, dc.bias, padding=1), rtol=1e-4, atol=1e-5)
    # a whole-pixel offset equals the convolution of the shifted input (interior outputs)
    off2 = off.clone()
    off2[:, 1::2] = 1.0  # dx = +1 for every tap
    shifted = F.conv2d(torch.cat([x[..., 1:], torch.zeros_like(x[..., :1])], -1), dc.weight, dc.bias, padding=1)
    torch.testing.assert_close(dc(x, off2)[..., 1:-2], shifted[..., 1:-2], rtol=1e-4, atol=1e-5)


def test_blocks_backbones_shuffle_segmetrics():
    for name, chans in (("resnet18", [64, 128, 256, 512]), ("resnet50", [256, 512, 1024, 2048])):
        bb = CX.BackboneZoo(name, base=64).eval()
        feats = bb.extract_features(torch.randn(1, 3, 64, 64))
        assert [f.shape[1] for f in feats] == chans == bb.out_channels
        assert [f.shape[-1] for f in feats] == [16, 8, 4, 2]
    x = torch.arange(8.0).view(1, 8, 1, 1)
    assert CX.channel_shuffle(x, 2).view(-1).tolist() == [0, 4, 1, 5, 2, 6, 3, 7]
    m = CX.SegMetrics(3, ignore_index=255)
    m.update(torch.tensor([0, 1, 1, 2]), torch.tensor([0, 1, 2, 255]))
    assert m.pixel_accuracy() == pytest.approx(2 / 3)
    assert m.iou().tolist()[:2] == [1.0, 0.5] and m.mean_iou() == pytest.approx((1.0 + 0.5 + 0.0) / 3)
    assert m.dice()[1].item() == pytest.approx(2 / 3)
