"""Computer-vision operators and blocks: box arithmetic, photometric and colour-space transforms,
geometric augmentation, RoI pooling, deformable convolution, residual/bottleneck blocks and a backbone
zoo, channel shuffle, segmentation metrics.

Reference: crates/brain-cv/src/ops/boxes.rs (box_area, box_iou_matrix, box_giou_matrix), ops/geometry.rs
(affine_grid, grid_sample), ops/hist_eq.rs (ColorSpace, equalize_histogram), augmentation/photo.rs
(solarize, equalize), augmentation/color.rs (ColorJitter), augmentation/boxes.rs
(transform_bounding_boxes), augmentation/geom.rs (RandomResizedCrop, Compose), detection/roi.rs
(RoIPool), conv/deformable.rs (DeformableConv2d), conv/residual.rs (BasicBlock, BottleneckBlock),
feature/backbones.rs (BackboneZoo), segmentation metrics and losses.

Several of these are placeholders in the reference (RoIPool returns zeros, deformable convolution
returns zeros, solarize/equalize/grid_sample return their input); here each computes its operation.
Images are [B, C, H, W] (or [C, H, W]) float tensors in [0, 1] on any device; everything is batched.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


# ------------------------------------------------------------------------------------------ boxes
def box_area(boxes: torch.Tensor) -> torch.Tensor:
    """[N, 4] xyxy -> [N] areas with negative extents clamped to 0."""
    return (boxes[:, 2] - boxes[:, 0]).clamp_min(0) * (boxes[:, 3] - boxes[:, 1]).clamp_min(0)


def _inter_union(a, b):
    lt = torch.maximum(a[:, None, :2], b[None, :, :2])
    rb = torch.minimum(a[:, None, 2:], b[None, :, 2:])
    inter = (rb - lt).clamp_min(0).prod(-1)
    union = box_area(a)[:, None] + box_area(b)[None, :] - inter
    return inter, union


def box_iou_matrix(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    inter, union = _inter_union(a, b)
    return torch.where(union > 0, inter / union.clamp_min(1e-300), torch.zeros_like(inter))


def box_giou_matrix(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """IoU minus the empty fraction of the smallest enclosing box (IoU itself when that box is empty)."""
    inter, union = _inter_union(a, b)
    iou = torch.where(union > 0, inter / union.clamp_min(1e-300), torch.zeros_like(inter))
    lt = torch.minimum(a[:, None, :2], b[None, :, :2])
    rb = torch.maximum(a[:, None, 2:], b[None, :, 2:])
    enc = (rb - lt).clamp_min(0).prod(-1)
    return torch.where(enc > 0, iou - (enc - union) / enc.clamp_min(1e-300), iou)


class BBoxFormat:
    XYXY, XYWH, CXCYWH = "xyxy", "xywh", "cxcywh"


def convert_bbox_format(boxes: torch.Tensor, src: str, dst: str) -> torch.Tensor:
    """Convert [N, 4] boxes between corner (xyxy), corner+size (xywh) and centre+size (cxcywh)."""
    if src == dst:
        return boxes.clone()
    x1, y1, a, b = boxes.unbind(-1)
    if src == BBoxFormat.XYWH:
        xyxy = torch.stack([x1, y1, x1 + a, y1 + b], -1)
    elif src == BBoxFormat.CXCYWH:
        xyxy = torch.stack([x1 - a / 2, y1 - b / 2, x1 + a / 2, y1 + b / 2], -1)
    else:
        xyxy = boxes
    X1, Y1, X2, Y2 = xyxy.unbind(-1)
    if dst == BBoxFormat.XYXY:
        return xyxy.clone()
    if dst == BBoxFormat.XYWH:
        return torch.stack([X1, Y1, X2 - X1, Y2 - Y1], -1)
    return torch.stack([(X1 + X2) / 2, (Y1 + Y2) / 2, X2 - X1, Y2 - Y1], -1)


def transform_bounding_boxes(boxes: torch.Tensor, img_w: float, flip_horizontal: bool) -> torch.Tensor:
    """xyxy boxes under a horizontal flip of an image of width img_w: x -> img_w - x (corners swap)."""
    if not flip_horizontal:
        return boxes.clone()
    return torch.stack([img_w - boxes[:, 2], boxes[:, 1], img_w - boxes[:, 0], boxes[:, 3]], -1)


def smooth_l1_loss(pred: torch.Tensor, target: torch.Tensor, beta: float = 1.0) -> torch.Tensor:
    return F.smooth_l1_loss(pred, target, beta=beta)


# ------------------------------------------------------------------------------------------ photometric
def solarize(image: torch.Tensor, threshold: float) -> torch.Tensor:
    """Invert (1 - x) every value at or above the threshold."""
    return torch.where(image >= threshold, 1.0 - image, image)


def equalize(image: torch.Tensor, bins: int = 256) -> torch.Tensor:
    """Per-image, per-channel histogram equalisation of [*, H, W] values in [0, 1]: each value maps to the
    normalised cumulative histogram of its bin (the lowest occupied bin maps to 0)."""
    shp = image.shape
    x = image.reshape(-1, shp[-2] * shp[-1])
    q = (x.clamp(0, 1) * (bins - 1)).round().long()
    hist = torch.zeros(x.shape[0], bins, device=x.device, dtype=torch.float64).scatter_add_(
        1, q, torch.ones_like(q, dtype=torch.float64))
    cdf = hist.cumsum(1)
    cmin = torch.where(hist > 0, cdf, torch.full_like(cdf, float("inf"))).min(1, keepdim=True).values
    total = cdf[:, -1:]
    lut = ((cdf - cmin) / (total - cmin).clamp_min(1.0)).clamp(0, 1)
    return lut.gather(1, q).to(image.dtype).reshape(shp)


equalize_histogram = equalize


class ColorSpace:
    RGB, HSV, LAB, YUV, GRAYSCALE = "rgb", "hsv", "lab", "yuv", "grayscale"


def rgb_to_gray(img: torch.Tensor) -> torch.Tensor:
    """ITU-R BT.601 luma, keeping a channel dimension of 1."""
    r, g, b = img.unbind(-3)
    return (0.299 * r + 0.587 * g + 0.114 * b).unsqueeze(-3)


def rgb_to_yuv(img: torch.Tensor) -> torch.Tensor:
    r, g, b = img.unbind(-3)
    y = 0.299 * r + 0.587 * g + 0.114 * b
    return torch.stack([y, 0.492 * (b - y), 0.877 * (r - y)], -3)


def yuv_to_rgb(img: torch.Tensor) -> torch.Tensor:
    y, u, v = img.unbind(-3)
    b = y + u / 0.492
    r = y + v / 0.877
    g = (y - 0.299 * r - 0.114 * b) / 0.587
    return torch.stack([r, g, b], -3)


def rgb_to_hsv(img: torch.Tensor) -> torch.Tensor:
    """Hue in [0, 1) (fraction of a turn), saturation and value in [0, 1]."""
    r, g, b = img.unbind(-3)
    mx, _ = img.max(-3)
    mn, _ = img.min(-3)
    d = mx - mn
    safe = torch.where(d > 0, d, torch.ones_like(d))
    h = torch.where(mx == r, ((g - b) / safe) % 6, torch.where(mx == g, (b - r) / safe + 2, (r - g) / safe + 4)) / 6
    h = torch.where(d > 0, h, torch.zeros_like(h))
    s = torch.where(mx > 0, d / torch.where(mx > 0, mx, torch.ones_like(mx)), torch.zeros_like(mx))
    return torch.stack([h % 1.0, s, mx], -3)


def hsv_to_rgb(img: torch.Tensor) -> torch.Tensor:
    h, s, v = img.unbind(-3)
    k = lambda n: (n + h * 6) % 6  # noqa: E731
    f = lambda n: v - v * s * torch.clamp(torch.minimum(k(n), 4 - k(n)), 0, 1)  # noqa: E731
    return torch.stack([f(5), f(3), f(1)], -3)


def rgb_to_lab(img: torch.Tensor) -> torch.Tensor:
    """sRGB (D65) -> CIE L*a*b*: linearise, to XYZ, normalise by the white point, cube-root companding."""
    lin = torch.where(img > 0.04045, ((img + 0.055) / 1.055) ** 2.4, img / 12.92)
    r, g, b = lin.unbind(-3)
    x = (0.4124564 * r + 0.3575761 * g + 0.1804375 * b) / 0.95047
    y = 0.2126729 * r + 0.7151522 * g + 0.0721750 * b
    z = (0.0193339 * r + 0.1191920 * g + 0.9503041 * b) / 1.08883
    d = 6.0 / 29.0
    fx, fy, fz = (torch.where(t > d ** 3, t.clamp_min(1e-12) ** (1 / 3), t / (3 * d * d) + 4 / 29) for t in (x, y, z))
    return torch.stack([116 * fy - 16, 500 * (fx - fy), 200 * (fy - fz)], -3)


def convert_color(img: torch.Tensor, src: str, dst: str) -> torch.Tensor:
    if src == dst:
        return img.clone()
    rgb = {ColorSpace.RGB: lambda t: t, ColorSpace.HSV: hsv_to_rgb, ColorSpace.YUV: yuv_to_rgb}[src](img)
    return {ColorSpace.RGB: lambda t: t, ColorSpace.HSV: rgb_to_hsv, ColorSpace.YUV: rgb_to_yuv,
            ColorSpace.LAB: rgb_to_lab, ColorSpace.GRAYSCALE: rgb_to_gray}[dst](rgb)


class ColorJitter:
    """Random brightness, contrast, saturation (factors in [1 - p, 1 + p]) and hue shift (in
    [-hue, hue] turns), applied in that order per image."""

    def __init__(self, brightness=0.0, contrast=0.0, saturation=0.0, hue=0.0, generator=None):
        self.b, self.c, self.s, self.h, self.g = brightness, contrast, saturation, hue, generator

    def _f(self, p, n, dev):
        return 1.0 + (torch.rand(n, generator=self.g) * 2 - 1).to(dev) * p

    def apply(self, image: torch.Tensor) -> torch.Tensor:
        x = image if image.dim() == 4 else image[None]
        n, dev = x.shape[0], x.device
        v = lambda t: t.view(n, 1, 1, 1)  # noqa: E731
        if self.b:
            x = x * v(self._f(self.b, n, dev))
        if self.c:
            m = rgb_to_gray(x).mean((1, 2, 3), keepdim=True)
            x = (x - m) * v(self._f(self.c, n, dev)) + m
        if self.s:
            gray = rgb_to_gray(x)
            x = (x - gray) * v(self._f(self.s, n, dev)) + gray
        x = x.clamp(0, 1)
        if self.h:
            hsv = rgb_to_hsv(x)
            shift = ((torch.rand(n, generator=self.g) * 2 - 1) * self.h).to(dev)
            hsv = torch.stack([(hsv[:, 0] + shift.view(n, 1, 1)) % 1.0, hsv[:, 1], hsv[:, 2]], 1)
            x = hsv_to_rgb(hsv)
        return x if image.dim() == 4 else x[0]

    __call__ = apply


# ------------------------------------------------------------------------------------------ geometry
def affine_grid(theta: torch.Tensor, size, align_corners: bool = False) -> torch.Tensor:
    """Sampling grid [B, H, W, 2] in normalised coordinates for affine maps theta [B, 2, 3]."""
    return F.affine_grid(theta, list(size), align_corners=align_corners)


def grid_sample(inp: torch.Tensor, grid: torch.Tensor, mode: str = "bilinear", padding_mode: str = "zeros",
                align_corners: bool = False) -> torch.Tensor:
    return F.grid_sample(inp, grid, mode=mode, padding_mode=padding_mode, align_corners=align_corners)


class RandomResizedCrop:
    """Crop a random area fraction in ``scale`` with aspect ratio (log-uniform) in ``ratio`` and resize it
    to ``size`` (bilinear); falls back to a central crop after 10 tries."""

    def __init__(self, size, scale=(0.08, 1.0), ratio=(3 / 4, 4 / 3), seed: int = 0):
        self.size = (size, size) if isinstance(size, int) else tuple(size)
        self.scale, self.ratio, self.rng = scale, ratio, random.Random(seed)

    def params(self, h: int, w: int):
        area = h * w
        for _ in range(10):
            ta = area * self.rng.uniform(*self.scale)
            ar = math.exp(self.rng.uniform(math.log(self.ratio[0]), math.log(self.ratio[1])))
            cw, ch = int(round(math.sqrt(ta * ar))), int(round(math.sqrt(ta / ar)))
            if 0 < cw <= w and 0 < ch <= h:
                return self.rng.randint(0, h - ch), self.rng.randint(0, w - cw), ch, cw
        s = min(h, w)
        return (h - s) // 2, (w - s) // 2, s, s

    def __call__(self, img: torch.Tensor) -> torch.Tensor:
        x = img if img.dim() == 4 else img[None]
        t, l, ch, cw = self.params(x.shape[-2], x.shape[-1])
        out = F.interpolate(x[..., t:t + ch, l:l + cw], size=self.size, mode="bilinear", align_corners=False)
        return out if img.dim() == 4 else out[0]


class Compose:
    def __init__(self, transforms):
        self.transforms = list(transforms)

    def __call__(self, x):
        for t in self.transforms:
            x = t(x)
        return x


# ------------------------------------------------------------------------------------------ RoI pooling
class RoIPool(nn.Module):
    """Fast R-CNN RoI max pooling: each RoI (batch_idx, x1, y1, x2, y2) in image coordinates is scaled by
    spatial_scale and rounded to feature cells; its output bin (i, j) is the max over the cells it covers
    (0 for an empty bin). Output [R, C, oh, ow]."""

    def __init__(self, output_size, spatial_scale: float = 1.0):
        super().__init__()
        self.oh, self.ow = (output_size, output_size) if isinstance(output_size, int) else output_size
        self.scale = spatial_scale

    def forward(self, features: torch.Tensor, rois: torch.Tensor) -> torch.Tensor:
        B, C, H, W = features.shape
        R = rois.shape[0]
        out = features.new_zeros(R, C, self.oh, self.ow)
        if R == 0:
            return out
        b = rois[:, 0].long()
        x1 = torch.round(rois[:, 1] * self.scale).long()
        y1 = torch.round(rois[:, 2] * self.scale).long()
        x2 = torch.round(rois[:, 3] * self.scale).long()
        y2 = torch.round(rois[:, 4] * self.scale).long()
        rw = (x2 - x1 + 1).clamp_min(1).to(features.dtype)
        rh = (y2 - y1 + 1).clamp_min(1).to(features.dtype)
        ys = torch.arange(H, device=features.device)
        xs = torch.arange(W, device=features.device)
        for i in range(self.oh):
            hs = (y1 + torch.floor(i * rh / self.oh).long()).clamp(0, H)
            he = (y1 + torch.ceil((i + 1) * rh / self.oh).long()).clamp(0, H)
            my = (ys[None] >= hs[:, None]) & (ys[None] < he[:, None])  # [R, H]
            for j in range(self.ow):
                ws = (x1 + torch.floor(j * rw / self.ow).long()).clamp(0, W)
                we = (x1 + torch.ceil((j + 1) * rw / self.ow).long()).clamp(0, W)
                mx = (xs[None] >= ws[:, None]) & (xs[None] < we[:, None])  # [R, W]
                m = my[:, :, None] & mx[:, None, :]  # [R, H, W]
                vals = torch.where(m[:, None], features[b], torch.full_like(features[b], float("-inf")))
                mxv = vals.amax((2, 3))
                out[:, :, i, j] = torch.where(torch.isfinite(mxv), mxv, torch.zeros_like(mxv))
        return out


# ------------------------------------------------------------------------------------------ convolutions / blocks
class DeformableConv2d(nn.Module):
    """Deformable convolution (Dai et al. 2017): each kernel tap k samples the input bilinearly at
    p + p_k + offset_k(p), offsets [B, 2K, H_out, W_out] as (dy, dx) pairs per tap, zeros outside."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int = 3, stride: int = 1, padding: int = 1,
                 bias: bool = True):
        super().__init__()
        self.k, self.stride, self.pad = kernel_size, stride, padding
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels, kernel_size, kernel_size))
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        self.bias = nn.Parameter(torch.zeros(out_channels)) if bias else None

    def forward(self, x: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
        B, C, H, W = x.shape
        k, s, p = self.k, self.stride, self.pad
        Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
        oy = (torch.arange(Ho, device=x.device) * s - p).to(x.dtype)
        ox = (torch.arange(Wo, device=x.device) * s - p).to(x.dtype)
        ky, kx = torch.meshgrid(torch.arange(k, device=x.device), torch.arange(k, device=x.device), indexing="ij")
        ky, kx = ky.reshape(-1).to(x.dtype), kx.reshape(-1).to(x.dtype)  # [K]
        off = offsets.view(B, k * k, 2, Ho, Wo)
        py = oy[None, None, :, None] + ky[None, :, None, None] + off[:, :, 0]  # [B, K, Ho, Wo]
        px = ox[None, None, None, :] + kx[None, :, None, None] + off[:, :, 1]
        grid = torch.stack([2 * px / max(W - 1, 1) - 1, 2 * py / max(H - 1, 1) - 1], -1)  # align_corners=True
        samp = F.grid_sample(x, grid.view(B, k * k * Ho, Wo, 2), mode="bilinear", padding_mode="zeros",
                             align_corners=True).view(B, C, k * k, Ho, Wo)
        out = torch.einsum("bckhw,ock->bohw", samp, self.weight.view(self.weight.shape[0], C, k * k))
        return out + self.bias.view(1, -1, 1, 1) if self.bias is not None else out


class BasicBlock(nn.Module):
    """ResNet basic block: two 3x3 conv-BN (ReLU between), projection shortcut on a shape change."""
    expansion = 1

    def __init__(self, cin: int, cout: int, stride: int = 1):
        super().__init__()
        self.c1, self.b1 = nn.Conv2d(cin, cout, 3, stride, 1, bias=False), nn.BatchNorm2d(cout)
        self.c2, self.b2 = nn.Conv2d(cout, cout, 3, 1, 1, bias=False), nn.BatchNorm2d(cout)
        self.short = (nn.Sequential(nn.Conv2d(cin, cout, 1, stride, bias=False), nn.BatchNorm2d(cout))
                      if stride != 1 or cin != cout else nn.Identity())

    def forward(self, x):
        return F.relu(self.b2(self.c2(F.relu(self.b1(self.c1(x))))) + self.short(x))


class BottleneckBlock(nn.Module):
    """1x1 reduce, 3x3 (strided), 1x1 expand by 4, with a projection shortcut on a shape change."""
    expansion = 4

    def __init__(self, cin: int, width: int, stride: int = 1):
        super().__init__()
        cout = width * 4
        self.c1, self.b1 = nn.Conv2d(cin, width, 1, bias=False), nn.BatchNorm2d(width)
        self.c2, self.b2 = nn.Conv2d(width, width, 3, stride, 1, bias=False), nn.BatchNorm2d(width)
        self.c3, self.b3 = nn.Conv2d(width, cout, 1, bias=False), nn.BatchNorm2d(cout)
        self.short = (nn.Sequential(nn.Conv2d(cin, cout, 1, stride, bias=False), nn.BatchNorm2d(cout))
                      if stride != 1 or cin != cout else nn.Identity())

    def forward(self, x):
        h = F.relu(self.b1(self.c1(x)))
        h = F.relu(self.b2(self.c2(h)))
        return F.relu(self.b3(self.c3(h)) + self.short(x))


class BackboneZoo(nn.Module):
    """ResNet-18/34/50-style backbones; ``extract_features`` returns the four stage outputs (strides 4,
    8, 16, 32 relative to the input), ``num_stages`` is 4."""

    LAYOUTS = {"resnet18": (BasicBlock, (2, 2, 2, 2)), "resnet34": (BasicBlock, (3, 4, 6, 3)),
               "resnet50": (BottleneckBlock, (3, 4, 6, 3))}

    def __init__(self, name: str = "resnet18", in_channels: int = 3, base: int = 64):
        super().__init__()
        self.name, self.num_stages = name, 4
        block, counts = self.LAYOUTS[name]
        self.stem = nn.Sequential(nn.Conv2d(in_channels, base, 7, 2, 3, bias=False), nn.BatchNorm2d(base), nn.ReLU(),
                                  nn.MaxPool2d(3, 2, 1))
        stages, cin = [], base
        for i, n in enumerate(counts):
            width = base * 2 ** i
            layers = []
            for j in range(n):
                layers.append(block(cin, width, 2 if (j == 0 and i > 0) else 1))
                cin = width * block.expansion
            stages.append(nn.Sequential(*layers))
        self.stages = nn.ModuleList(stages)
        self.out_channels = [base * 2 ** i * block.expansion for i in range(4)]

    @classmethod
    def resnet50(cls, **kw):
        return cls("resnet50", **kw)

    def extract_features(self, x: torch.Tensor):
        h = self.stem(x)
        feats = []
        for st in self.stages:
            h = st(h)
            feats.append(h)
        return feats

    forward = extract_features


def channel_shuffle(x: torch.Tensor, groups: int) -> torch.Tensor:
    """[B, g * c, H, W] -> interleave the groups' channels (ShuffleNet)."""
    B, C, H, W = x.shape
    return x.view(B, groups, C // groups, H, W).transpose(1, 2).reshape(B, C, H, W)


# ------------------------------------------------------------------------------------------ segmentation
class SegMetrics:
    """Streaming confusion matrix over batches of label maps: pixel accuracy, per-class and mean IoU,
    per-class Dice; ``ignore_index`` pixels are skipped."""

    def __init__(self, num_classes: int, ignore_index: int = -1, device=None):
        self.k, self.ignore = num_classes, ignore_index
        self.cm = torch.zeros(num_classes, num_classes, dtype=torch.long, device=device)

    def update(self, pred: torch.Tensor, target: torch.Tensor) -> None:
        p, t = pred.reshape(-1).long(), target.reshape(-1).long()
        keep = (t != self.ignore) & (t >= 0) & (t < self.k)
        idx = t[keep] * self.k + p[keep].clamp(0, self.k - 1)
        self.cm += torch.bincount(idx, minlength=self.k * self.k).view(self.k, self.k).to(self.cm.device)

    def pixel_accuracy(self) -> float:
        tot = int(self.cm.sum())
        return float(self.cm.diag().sum()) / tot if tot else 0.0

    def iou(self) -> torch.Tensor:
        tp = self.cm.diag().double()
        den = self.cm.sum(0).double() + self.cm.sum(1).double() - tp
        return torch.where(den > 0, tp / den.clamp_min(1), torch.full_like(tp, float("nan")))

    def mean_iou(self) -> float:
        v = self.iou()
        return float(v[~torch.isnan(v)].mean()) if bool((~torch.isnan(v)).any()) else 0.0

    def dice(self) -> torch.Tensor:
        tp = self.cm.diag().double()
        den = self.cm.sum(0).double() + self.cm.sum(1).double()
        return torch.where(den > 0, 2 * tp / den.clamp_min(1), torch.full_like(tp, float("nan")))


# ------------------------------------------------------------------ MobileNetV3 (Howard et al. 2019), small / large
# crates/brain-cv/src/feature/backbones.rs (mobilenet_v3). Inverted residual blocks: 1x1 expansion,
# depthwise k x k (stride s), optional squeeze-excitation (hard-sigmoid gate), 1x1 projection,
# residual when the shape is kept; hard-swish or ReLU per block.

class _SqueezeExcite(torch.nn.Module):
    def __init__(self, c: int, r: int = 4):
        super().__init__()
        m = max(8, c // r)
        self.fc1, self.fc2 = torch.nn.Conv2d(c, m, 1), torch.nn.Conv2d(m, c, 1)

    def forward(self, x):
        s = F.adaptive_avg_pool2d(x, 1)
        return x * F.hardsigmoid(self.fc2(F.relu(self.fc1(s))))


class InvertedResidual(torch.nn.Module):
    def __init__(self, cin: int, k: int, exp: int, cout: int, se: bool, act: str, stride: int):
        super().__init__()
        a = torch.nn.Hardswish if act == "hs" else torch.nn.ReLU
        layers = []
        if exp != cin:
            layers += [torch.nn.Conv2d(cin, exp, 1, bias=False), torch.nn.BatchNorm2d(exp), a()]
        layers += [torch.nn.Conv2d(exp, exp, k, stride, k // 2, groups=exp, bias=False), torch.nn.BatchNorm2d(exp), a()]
        if se:
            layers.append(_SqueezeExcite(exp))
        layers += [torch.nn.Conv2d(exp, cout, 1, bias=False), torch.nn.BatchNorm2d(cout)]
        self.block = torch.nn.Sequential(*layers)
        self.residual = stride == 1 and cin == cout

    def forward(self, x):
        y = self.block(x)
        return x + y if self.residual else y


_MBV3 = {  # (kernel, expansion, out, squeeze-excite, activation, stride)
    "small": [(3, 16, 16, True, "re", 2), (3, 72, 24, False, "re", 2), (3, 88, 24, False, "re", 1),
              (5, 96, 40, True, "hs", 2), (5, 240, 40, True, "hs", 1), (5, 240, 40, True, "hs", 1),
              (5, 120, 48, True, "hs", 1), (5, 144, 48, True, "hs", 1), (5, 288, 96, True, "hs", 2),
              (5, 576, 96, True, "hs", 1), (5, 576, 96, True, "hs", 1)],
    "large": [(3, 16, 16, False, "re", 1), (3, 64, 24, False, "re", 2), (3, 72, 24, False, "re", 1),
              (5, 72, 40, True, "re", 2), (5, 120, 40, True, "re", 1), (5, 120, 40, True, "re", 1),
              (3, 240, 80, False, "hs", 2), (3, 200, 80, False, "hs", 1), (3, 184, 80, False, "hs", 1),
              (3, 184, 80, False, "hs", 1), (3, 480, 112, True, "hs", 1), (3, 672, 112, True, "hs", 1),
              (5, 672, 160, True, "hs", 2), (5, 960, 160, True, "hs", 1), (5, 960, 160, True, "hs", 1)],
}


class MobileNetV3(torch.nn.Module):
    """``variant`` small or large; ``width`` scales every channel count (rounded to multiples of 8)."""

    def __init__(self, num_classes: int = 1000, variant: str = "small", width: float = 1.0, in_channels: int = 3):
        super().__init__()

        def c(v):
            return max(8, int(v * width + 4) // 8 * 8)
        layers = [torch.nn.Conv2d(in_channels, c(16), 3, 2, 1, bias=False), torch.nn.BatchNorm2d(c(16)),
                  torch.nn.Hardswish()]
        cin = c(16)
        for k, e, o, se, act, s in _MBV3[variant]:
            layers.append(InvertedResidual(cin, k, c(e), c(o), se, act, s))
            cin = c(o)
        last = c(576 if variant == "small" else 960)
        layers += [torch.nn.Conv2d(cin, last, 1, bias=False), torch.nn.BatchNorm2d(last), torch.nn.Hardswish()]
        self.features = torch.nn.Sequential(*layers)
        hidden = 1024 if variant == "small" else 1280
        self.classifier = torch.nn.Sequential(torch.nn.Linear(last, hidden), torch.nn.Hardswish(),
                                              torch.nn.Dropout(0.2), torch.nn.Linear(hidden, num_classes))
        self.out_channels = last

    def forward_features(self, x):
        return self.features(x)

    def forward(self, x):
        return self.classifier(F.adaptive_avg_pool2d(self.features(x), 1).flatten(1))


def mobilenet_v3(num_classes: int = 1000, variant: str = "small", width: float = 1.0) -> MobileNetV3:
    return MobileNetV3(num_classes, variant, width)
