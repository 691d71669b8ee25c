"""Computer vision: convolution blocks (depthwise-separable, grouped, ghost, weight-standardised,
residual), a small ResNet backbone with a feature pyramid, image augmentation (flips, crops, colour
jitter, mixup, cutmix), detection utilities (box formats, IoU, anchors, box coding, NMS) and a
fully-convolutional segmentation head with Dice loss.

Reference: crates/brain-cv. Convs (conv/depthwise.rs, conv/grouped.rs, conv/ghost.rs, conv/ws.rs,
conv/residual.rs), backbones and FPN (feature/backbones.rs, feature/fpn.rs), augmentation
(augmentation/geom.rs, color.rs, mix.rs), detection (detection/anchor.rs:9-60,
detection/postprocess.rs:9-80, detection/roi.rs), segmentation (segmentation/fcn.rs, losses.rs).

Convolutions run on cuDNN through PyTorch (no custom kernel is planned for them); batched box math
and NMS are tensor ops on the boxes' device.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..nn.module import Module


class DepthwiseSeparableConv(Module):
    def __init__(self, cin, cout, k=3, stride=1, device=None, dtype=None):
        super().__init__()
        self.dw = torch.nn.Conv2d(cin, cin, k, stride, k // 2, groups=cin, bias=False, device=device, dtype=dtype)
        self.pw = torch.nn.Conv2d(cin, cout, 1, bias=False, device=device, dtype=dtype)
        self.bn = torch.nn.BatchNorm2d(cout, device=device, dtype=dtype)

    def forward(self, x):
        return F.relu(self.bn(self.pw(self.dw(x))))


class GroupedConv(Module):
    def __init__(self, cin, cout, k=3, groups=4, stride=1, device=None, dtype=None):
        super().__init__()
        self.conv = torch.nn.Conv2d(cin, cout, k, stride, k // 2, groups=groups, bias=False, device=device, dtype=dtype)

    def forward(self, x):
        return self.conv(x)


class GhostConv(Module):
    """Half the output channels from a regular conv, the other half from a cheap depthwise conv of them."""

    def __init__(self, cin, cout, k=1, dw_k=3, device=None, dtype=None):
        super().__init__()
        half = cout // 2
        self.primary = torch.nn.Conv2d(cin, half, k, 1, k // 2, bias=False, device=device, dtype=dtype)
        self.cheap = torch.nn.Conv2d(half, cout - half, dw_k, 1, dw_k // 2, groups=half if (cout - half) % half == 0
                                     else 1, bias=False, device=device, dtype=dtype)

    def forward(self, x):
        y = self.primary(x)
        return torch.cat([y, self.cheap(y)], 1)


class WSConv2d(torch.nn.Conv2d):
    """Weight standardisation: each filter normalised to zero mean, unit variance before the conv."""

    def forward(self, x):
        w = self.weight
        m = w.mean(dim=(1, 2, 3), keepdim=True)
        v = w.var(dim=(1, 2, 3), keepdim=True, unbiased=False)
        return F.conv2d(x, (w - m) / torch.sqrt(v + 1e-5), self.bias, self.stride, self.padding, self.dilation,
                        self.groups)


class ResidualBlock(Module):
    def __init__(self, cin, cout, stride=1, device=None, dtype=None):
        super().__init__()
        self.c1 = torch.nn.Conv2d(cin, cout, 3, stride, 1, bias=False, device=device, dtype=dtype)
        self.b1 = torch.nn.BatchNorm2d(cout, device=device, dtype=dtype)
        self.c2 = torch.nn.Conv2d(cout, cout, 3, 1, 1, bias=False, device=device, dtype=dtype)
        self.b2 = torch.nn.BatchNorm2d(cout, device=device, dtype=dtype)
        self.skip = (torch.nn.Sequential(torch.nn.Conv2d(cin, cout, 1, stride, bias=False, device=device, dtype=dtype),
                                         torch.nn.BatchNorm2d(cout, device=device, dtype=dtype))
                     if stride != 1 or cin != cout else torch.nn.Identity())

    def forward(self, x):
        return F.relu(self.b2(self.c2(F.relu(self.b1(self.c1(x))))) + self.skip(x))


class ResNetLite(Module):
    """Stem + stages of residual blocks (stride 2 between stages); ``features`` returns each stage's map."""

    def __init__(self, in_ch=3, widths=(32, 64, 128), blocks=(1, 1, 1), num_classes=10, device=None, dtype=None):
        super().__init__()
        self.stem = torch.nn.Sequential(torch.nn.Conv2d(in_ch, widths[0], 3, 1, 1, bias=False, device=device, dtype=dtype),
                                        torch.nn.BatchNorm2d(widths[0], device=device, dtype=dtype), torch.nn.ReLU())
        stages, c = [], widths[0]
        for i, (w, n) in enumerate(zip(widths, blocks)):
            layers = [ResidualBlock(c, w, 1 if i == 0 else 2, device, dtype)]
            layers += [ResidualBlock(w, w, 1, device, dtype) for _ in range(n - 1)]
            stages.append(torch.nn.Sequential(*layers))
            c = w
        self.stages = torch.nn.ModuleList(stages)
        self.fc = torch.nn.Linear(c, num_classes, device=device, dtype=dtype)
        self.widths = widths

    def features(self, x):
        x = self.stem(x)
        out = []
        for s in self.stages:
            x = s(x)
            out.append(x)
        return out

    def forward(self, x):
        return self.fc(self.features(x)[-1].mean((2, 3)))


class FPN(Module):
    """Top-down feature pyramid: lateral 1x1 convs, nearest upsampling + add, 3x3 smoothing."""

    def __init__(self, in_channels, out_ch=64, device=None, dtype=None):
        super().__init__()
        self.lat = torch.nn.ModuleList([torch.nn.Conv2d(c, out_ch, 1, device=device, dtype=dtype) for c in in_channels])
        self.smooth = torch.nn.ModuleList([torch.nn.Conv2d(out_ch, out_ch, 3, 1, 1, device=device, dtype=dtype)
                                           for _ in in_channels])

    def forward(self, feats):
        lat = [l(f) for l, f in zip(self.lat, feats)]
        out = [lat[-1]]
        for f in reversed(lat[:-1]):
            out.insert(0, f + F.interpolate(out[0], size=f.shape[-2:], mode="nearest"))
        return [s(o) for s, o in zip(self.smooth, out)]


# ------------------------------------------------------------------ augmentation
def random_horizontal_flip(img, p=0.5, generator=None):
    if float(torch.rand(1, generator=generator)) < p:
        return img.flip(-1)
    return img


def random_crop(img, size, padding=0, generator=None):
    if padding:
        img = F.pad(img, (padding,) * 4)
    H, W = img.shape[-2:]
    th, tw = size
    y = int(torch.randint(0, H - th + 1, (1,), generator=generator))
    x = int(torch.randint(0, W - tw + 1, (1,), generator=generator))
    return img[..., y:y + th, x:x + tw]


def color_jitter(img, brightness=0.2, contrast=0.2, saturation=0.2, generator=None):
    def f(s):
        return 1 + (float(torch.rand(1, generator=generator)) * 2 - 1) * s

    out = img * f(brightness)
    m = out.mean(dim=(-3, -2, -1), keepdim=True)
    out = (out - m) * f(contrast) + m
    if img.shape[-3] == 3:
        gray = (0.299 * out[..., 0:1, :, :] + 0.587 * out[..., 1:2, :, :] + 0.114 * out[..., 2:3, :, :])
        out = (out - gray) * f(saturation) + gray
    return out


def mixup(x, y_onehot, alpha=0.2, generator=None):
    lam = float(torch.distributions.Beta(alpha, alpha).sample()) if alpha > 0 else 1.0
    perm = torch.randperm(x.shape[0], generator=generator).to(x.device)
    return lam * x + (1 - lam) * x[perm], lam * y_onehot + (1 - lam) * y_onehot[perm]


def cutmix(x, y_onehot, alpha=1.0, generator=None):
    lam = float(torch.distributions.Beta(alpha, alpha).sample()) if alpha > 0 else 1.0
    H, W = x.shape[-2:]
    rh, rw = int(H * (1 - lam) ** 0.5), int(W * (1 - lam) ** 0.5)
    cy = int(torch.randint(0, H, (1,), generator=generator))
    cx = int(torch.randint(0, W, (1,), generator=generator))
    y0, y1, x0, x1 = max(cy - rh // 2, 0), min(cy + rh // 2, H), max(cx - rw // 2, 0), min(cx + rw // 2, W)
    perm = torch.randperm(x.shape[0], generator=generator).to(x.device)
    out = x.clone()
    out[..., y0:y1, x0:x1] = x[perm][..., y0:y1, x0:x1]
    lam_adj = 1 - (y1 - y0) * (x1 - x0) / (H * W)
    return out, lam_adj * y_onehot + (1 - lam_adj) * y_onehot[perm]


# ------------------------------------------------------------------ detection
def xyxy_to_cxcywh(b):
    return torch.stack([(b[..., 0] + b[..., 2]) / 2, (b[..., 1] + b[..., 3]) / 2, b[..., 2] - b[..., 0],
                        b[..., 3] - b[..., 1]], -1)


def cxcywh_to_xyxy(b):
    return torch.stack([b[..., 0] - b[..., 2] / 2, b[..., 1] - b[..., 3] / 2, b[..., 0] + b[..., 2] / 2,
                        b[..., 1] + b[..., 3] / 2], -1)


def compute_iou(a, b):
    """Pairwise IoU of xyxy boxes: [N, 4] x [M, 4] -> [N, M]."""
    area = lambda t: (t[:, 2] - t[:, 0]).clamp(min=0) * (t[:, 3] - t[:, 1]).clamp(min=0)  # noqa: E731
    lt = torch.maximum(a[:, None, :2], b[None, :, :2])
    rb = torch.minimum(a[:, None, 2:], b[None, :, 2:])
    inter = (rb - lt).clamp(min=0).prod(-1)
    return inter / (area(a)[:, None] + area(b)[None] - inter + 1e-12)


def nms(boxes, scores, iou_threshold=0.5):
    """Greedy non-maximum suppression; returns kept indices in descending score order."""
    order = scores.argsort(descending=True)
    iou = compute_iou(boxes, boxes)
    keep, suppressed = [], torch.zeros(boxes.shape[0], dtype=torch.bool, device=boxes.device)
    for i in order.tolist():
        if suppressed[i]:
            continue
        keep.append(i)
        suppressed |= iou[i] > iou_threshold
    return torch.tensor(keep, dtype=torch.long, device=boxes.device)


class AnchorGenerator:
    def __init__(self, scales=(32.0,), aspect_ratios=(0.5, 1.0, 2.0)):
        self.scales, self.aspect_ratios = list(scales), list(aspect_ratios)

    def base_anchors(self):
        out = []
        for s in self.scales:
            for r in self.aspect_ratios:
                w, h = s / r ** 0.5, s * r ** 0.5
                out.append([-w / 2, -h / 2, w / 2, h / 2])
        return torch.tensor(out)

    def generate_grid_anchors(self, feat_h, feat_w, stride):
        """[feat_h * feat_w * A, 4] xyxy anchors centred on each cell."""
        ys = (torch.arange(feat_h) + 0.5) * stride
        xs = (torch.arange(feat_w) + 0.5) * stride
        cy, cx = torch.meshgrid(ys, xs, indexing="ij")
        ctr = torch.stack([cx, cy, cx, cy], -1).reshape(-1, 1, 4)
        return (ctr + self.base_anchors()[None]).reshape(-1, 4)


def encode_boxes(gt, anchors, weights=(10.0, 10.0, 5.0, 5.0)):
    """Faster R-CNN deltas (dx, dy, dw, dh) of xyxy ground truth relative to xyxy anchors."""
    g, a = xyxy_to_cxcywh(gt), xyxy_to_cxcywh(anchors)
    return torch.stack([weights[0] * (g[:, 0] - a[:, 0]) / a[:, 2], weights[1] * (g[:, 1] - a[:, 1]) / a[:, 3],
                        weights[2] * torch.log(g[:, 2] / a[:, 2]), weights[3] * torch.log(g[:, 3] / a[:, 3])], -1)


def decode_boxes(deltas, anchors, weights=(10.0, 10.0, 5.0, 5.0)):
    a = xyxy_to_cxcywh(anchors)
    cx = deltas[:, 0] / weights[0] * a[:, 2] + a[:, 0]
    cy = deltas[:, 1] / weights[1] * a[:, 3] + a[:, 1]
    w = torch.exp(deltas[:, 2] / weights[2]) * a[:, 2]
    h = torch.exp(deltas[:, 3] / weights[3]) * a[:, 3]
    return cxcywh_to_xyxy(torch.stack([cx, cy, w, h], -1))


def roi_align(feat, boxes, output_size=7, spatial_scale=1.0):
    """Bilinear ROI pooling: feat [C, H, W], boxes [K, 4] xyxy -> [K, C, S, S] (one sample per bin)."""
    K = boxes.shape[0]
    S = output_size
    b = boxes * spatial_scale
    t = (torch.arange(S, device=feat.device, dtype=feat.dtype) + 0.5) / S
    xs = b[:, 0:1] + t[None] * (b[:, 2:3] - b[:, 0:1])
    ys = b[:, 1:2] + t[None] * (b[:, 3:4] - b[:, 1:2])
    H, W = feat.shape[-2:]
    gx = xs / W * 2 - 1
    gy = ys / H * 2 - 1
    grid = torch.stack([gx[:, None, :].expand(K, S, S), gy[:, :, None].expand(K, S, S)], -1)
    return F.grid_sample(feat[None].expand(K, -1, -1, -1), grid, align_corners=False)


# ------------------------------------------------------------------ segmentation
class FcnHead(Module):
    def __init__(self, cin, num_classes, mid=64, device=None, dtype=None):
        super().__init__()
        self.c1 = torch.nn.Conv2d(cin, mid, 3, 1, 1, device=device, dtype=dtype)
        self.c2 = torch.nn.Conv2d(mid, num_classes, 1, device=device, dtype=dtype)

    def forward(self, feat, out_size):
        return F.interpolate(self.c2(F.relu(self.c1(feat))), size=out_size, mode="bilinear", align_corners=False)


def dice_loss(logits, target, eps=1.0):
    """Soft Dice over classes: logits [B, C, H, W], integer target [B, H, W]."""
    p = logits.softmax(1)
    t = F.one_hot(target, logits.shape[1]).permute(0, 3, 1, 2).to(p.dtype)
    inter = (p * t).sum((0, 2, 3))
    den = p.sum((0, 2, 3)) + t.sum((0, 2, 3))
    return 1 - ((2 * inter + eps) / (den + eps)).mean()


# ------------------------------------------------------------------ the reference's names
# crates/brain-cv/src: conv/{depthwise,grouped,ghost,ws}.rs, detection/{nms,roi_align}.rs, augmentation/mix.rs.
DepthwiseSeparableConv2d = DepthwiseSeparableConv
GroupedConv2d = GroupedConv
GhostModule = GhostConv
Conv2dWS = WSConv2d
non_max_suppression = nms


class RoIAlign(Module):
    """Module form of ``roi_align``: (feat [C, H, W], boxes [K, 4] xyxy) -> [K, C, S, S]."""

    def __init__(self, output_size: int = 7, spatial_scale: float = 1.0):
        super().__init__()
        self.output_size, self.spatial_scale = output_size, spatial_scale

    def forward(self, feat, boxes):
        return roi_align(feat, boxes, self.output_size, self.spatial_scale)


def sample_cutmix_box(H: int, W: int, lam: float, generator=None):
    """(y0, y1, x0, x1) of a box covering (1 - lam) of an H x W image, centred uniformly at random."""
    rh, rw = int(H * (1 - lam) ** 0.5), int(W * (1 - lam) ** 0.5)
    cy = int(torch.randint(0, H, (1,), generator=generator))
    cx = int(torch.randint(0, W, (1,), generator=generator))
    return max(cy - rh // 2, 0), min(cy + rh // 2, H), max(cx - rw // 2, 0), min(cx + rw // 2, W)
