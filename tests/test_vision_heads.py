"""ViT detection / segmentation heads, box and mask metrics, and backbones (crates/brain-vit/src/detection,
segmentation, backbones), with the reference tests' expectations."""
import math

import pytest
import torch

from brain_b200.models import vision as V


def test_bbox_geometry():
    b = V.Bbox(0.5, 0.5, 0.4, 0.6, 1.0, 0)
    assert all(abs(x - y) < 1e-9 for x, y in zip(b.to_xyxy(), [0.3, 0.2, 0.7, 0.8]))
    c = V.Bbox.from_xyxy(0.1, 0.2, 0.5, 0.7, 0.8, 1)
    assert abs(c.cx - 0.3) < 1e-9 and abs(c.cy - 0.45) < 1e-9
    assert abs(V.Bbox(0.5, 0.5, 0.2, 0.3).area() - 0.06) < 1e-10
    assert V.Bbox(0.5, 0.5, 2.0, 2.0).clamp().w <= 1.0
    assert "Bbox(" in str(b)


def test_iou_giou_nms():
    a = V.Bbox(0.5, 0.5, 0.2, 0.2)
    assert abs(V.iou(a, a) - 1.0) < 1e-12 and abs(V.giou(a, a) - 1.0) < 1e-12
    far = V.Bbox(0.9, 0.9, 0.1, 0.1)
    assert V.iou(a, far) == 0.0 and V.giou(a, far) < 0.0
    boxes = [V.Bbox(0.5, 0.5, 0.2, 0.2, 0.9, 0), V.Bbox(0.51, 0.5, 0.2, 0.2, 0.8, 0),
             V.Bbox(0.51, 0.5, 0.2, 0.2, 0.7, 1), V.Bbox(0.1, 0.1, 0.1, 0.1, 0.6, 0)]
    kept = V.nms(boxes, 0.5)
    assert [k.score for k in kept] == [0.9, 0.7, 0.6]  # the class-0 duplicate is suppressed, class 1 is not
    t = torch.tensor([[b.cx, b.cy, b.w, b.h] for b in boxes])
    idx = V.nms_tensor(t, torch.tensor([b.score for b in boxes]), torch.tensor([b.class_id for b in boxes]), 0.5)
    assert idx.tolist() == [0, 2, 3]
    m = V.box_iou_matrix(t, t)
    assert abs(float(m[0, 1]) - V.iou(boxes[0], boxes[1])) < 1e-6


def test_mean_average_precision():
    gt = [[V.Bbox(0.3, 0.3, 0.2, 0.2, 1, 0), V.Bbox(0.7, 0.7, 0.2, 0.2, 1, 1)]]
    assert abs(V.mean_average_precision(gt, gt, 0.5, 2) - 1.0) < 1e-9
    assert V.mean_average_precision([[]], gt, 0.5, 2) == 0.0
    half = [[V.Bbox(0.3, 0.3, 0.2, 0.2, 0.9, 0)]]
    assert abs(V.mean_average_precision(half, gt, 0.5, 2) - 0.5) < 1e-9


def test_detection_head_trains():
    torch.manual_seed(0)
    head = V.DetectionHead(16, 3, 5, seed=1)
    q = torch.randn(2, 5, 16)
    boxes, logits = head(q)
    assert boxes.shape == (2, 5, 4) and logits.shape == (2, 5, 4)
    assert float(boxes.min()) > 0 and float(boxes.max()) < 1
    assert head.num_params() == 4 * 16 + 4 + 4 * 16 + 4
    target_b, target_c = torch.rand(2, 5, 4), torch.randint(0, 4, (2, 5))
    opt = torch.optim.Adam(head.parameters(), lr=0.05)
    first = None
    for _ in range(60):
        b, c = head(q)
        loss = (b - target_b).abs().mean() + torch.nn.functional.cross_entropy(c.reshape(-1, 4), target_c.reshape(-1))
        first = float(loss) if first is None else first
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert float(loss) < 0.5 * first
    dec = head.decode_boxes(*head(q), score_threshold=0.0)
    assert len(dec) == 2 and len(dec[0]) == 5 and all(0 <= d.class_id < 3 for d in dec[0])
    with pytest.raises(ValueError):
        head(torch.randn(2, 4, 16))


def test_segmentation_decoder_and_metrics():
    dec = V.SegDecoder(8, 3, seed=2)
    logits = dec(torch.randn(2, 16, 8))
    assert logits.shape == (2, 16, 3) and V.SegDecoder.predict_class(logits).shape == (2, 16)
    preds, gts = [0, 1, 1, 2, 2, 2], [0, 1, 2, 2, 2, 0]
    ious, miou = V.per_class_iou(preds, gts, 3)
    assert abs(ious[0] - 0.5) < 1e-12 and abs(ious[1] - 0.5) < 1e-12 and abs(ious[2] - 0.5) < 1e-12
    assert abs(miou - 0.5) < 1e-12
    assert abs(V.pixel_accuracy(preds, gts) - 4 / 6) < 1e-12
    cm = V.confusion_matrix(preds, gts, 3)
    assert cm.sum() == 6 and cm[2, 1] == 1 and cm[0, 2] == 1
    assert V.dice_coefficient([True, False], [True, False]) == 1.0
    assert V.dice_coefficient([False], [False]) == 1.0
    assert abs(V.seg_iou_pair([True, True, False], [True, False, False]) - 0.5) < 1e-12
    ious, _ = V.per_class_iou([0, 0], [0, 0], 3)
    assert math.isnan(ious[1])
    up = V.UpscaleDecoder(8, 3, grid_size=4, out_h=32, out_w=32, seed=0)
    lg = up(torch.randn(2, 16, 8))
    assert up.upsample(lg).shape == (2, 3, 32, 32)


def test_backbones():
    bb = V.micro_backbone(seed=0)
    img = torch.randn(2, 1, 8, 8)
    f = bb.extract_features(img)
    assert f.shape == (2, 5, 16)
    assert bb.extract_cls(img).shape == (2, 16) and bb.extract_patches(img).shape == (2, 4, 16)
    assert bb.embed_dim() == 16 and bb.total_params() > 0
    bb.backbone_config.return_intermediate, bb.backbone_config.return_blocks = True, [0, 1]
    h, inter = bb.extract_features(img)
    assert len(inter) == 2 and inter[0].shape == (2, 5, 16)
    assert V.BackboneSize.Large.embed_dim() == 1024 and V.BackboneSize.Large.depth() == 24
    assert V.BackboneSize.Tiny.config().num_heads == 3
