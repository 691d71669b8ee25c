"""ViT task heads and backbones: object detection, semantic segmentation, feature extraction.

API parity with crates/brain-vit/src/detection/mod.rs (``Bbox``, ``iou``, ``giou``, ``nms``,
``DetectionHead`` with a sigmoid box regressor and a (classes + background) classifier per query,
``decode_boxes``, ``mean_average_precision``), crates/brain-vit/src/segmentation/mod.rs
(``SegDecoder`` per-patch linear classifier, ``predict_class``, ``per_class_iou``, ``pixel_accuracy``,
``confusion_matrix``, ``dice_coefficient``, ``UpscaleDecoder``, ``seg_iou_pair``) and
crates/brain-vit/src/backbones/mod.rs (``BackboneSize`` Tiny/Small/Base/Large, ``VitBackbone`` with
``extract_features`` / ``extract_cls`` / ``extract_patches``, ``micro_backbone``).

The heads are ``Module``s whose linears run on the framework's GEMM (tcgen05 on a B200, bf16), so they
train with autograd; box and mask metrics are host-side float64 like the reference's. Beyond the
reference: ``nms`` also takes batched tensors (``nms_tensor``, IoU matrix on the device), the
``UpscaleDecoder`` bilinearly resamples the patch-grid logits to the output size (``upsample``), and
``VitBackbone`` can return the hidden states of chosen blocks (``return_blocks``).
"""
from __future__ import annotations

import enum
import math
from dataclasses import dataclass, field

import torch

from ..nn.layers import Linear
from ..nn.module import Module
from .config import ViTConfig
from .families import ViT


# --------------------------------------------------------------------------- boxes
@dataclass
class Bbox:
    """Box in normalised centre form (cx, cy, w, h), with a score and a class id."""
    cx: float
    cy: float
    w: float
    h: float
    score: float = 1.0
    class_id: int = 0

    def to_xyxy(self):
        return [self.cx - self.w / 2, self.cy - self.h / 2, self.cx + self.w / 2, self.cy + self.h / 2]

    @staticmethod
    def from_xyxy(x1, y1, x2, y2, score=1.0, class_id=0) -> "Bbox":
        return Bbox((x1 + x2) / 2, (y1 + y2) / 2, x2 - x1, y2 - y1, score, class_id)

    def area(self) -> float:
        return self.w * self.h

    def clamp(self) -> "Bbox":
        c = lambda v: min(1.0, max(0.0, v))  # noqa: E731
        return Bbox(c(self.cx), c(self.cy), c(self.w), c(self.h), self.score, self.class_id)

    def __str__(self):
        return (f"Bbox(cx={self.cx:.3f}, cy={self.cy:.3f}, w={self.w:.3f}, h={self.h:.3f}, "
                f"cls={self.class_id}, score={self.score:.3f})")


def _inter_union(a: Bbox, b: Bbox):
    ax1, ay1, ax2, ay2 = a.to_xyxy()
    bx1, by1, bx2, by2 = b.to_xyxy()
    inter = max(0.0, min(ax2, bx2) - max(ax1, bx1)) * max(0.0, min(ay2, by2) - max(ay1, by1))
    return inter, a.area() + b.area() - inter, (ax1, ay1, ax2, ay2, bx1, by1, bx2, by2)


def iou(a: Bbox, b: Bbox) -> float:
    inter, union, _ = _inter_union(a, b)
    return 0.0 if union <= 0 else inter / union


def giou(a: Bbox, b: Bbox) -> float:
    """Generalised IoU: IoU minus the share of the enclosing box not covered by the union."""
    inter, union, (ax1, ay1, ax2, ay2, bx1, by1, bx2, by2) = _inter_union(a, b)
    v = 0.0 if union <= 0 else inter / union
    enc = (max(ax2, bx2) - min(ax1, bx1)) * (max(ay2, by2) - min(ay1, by1))
    return v if enc <= 0 else v - (enc - union) / enc


def nms(boxes: list[Bbox], iou_threshold: float) -> list[Bbox]:
    """Greedy per-class non-maximum suppression in descending score order (stable for ties)."""
    order = sorted(range(len(boxes)), key=lambda i: -boxes[i].score)
    kept, suppressed = [], [False] * len(order)
    for ii, i in enumerate(order):
        if suppressed[ii]:
            continue
        kept.append(boxes[i])
        for jj in range(ii + 1, len(order)):
            j = order[jj]
            if not suppressed[jj] and boxes[i].class_id == boxes[j].class_id and iou(boxes[i], boxes[j]) > iou_threshold:
                suppressed[jj] = True
    return kept


def box_iou_matrix(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """IoU of every pair of centre-form boxes a [N, 4], b [M, 4] -> [N, M] (on their device)."""
    def xyxy(t):
        return torch.stack([t[:, 0] - t[:, 2] / 2, t[:, 1] - t[:, 3] / 2, t[:, 0] + t[:, 2] / 2, t[:, 1] + t[:, 3] / 2], 1)
    A, B = xyxy(a.float()), xyxy(b.float())
    lt = torch.maximum(A[:, None, :2], B[None, :, :2])
    rb = torch.minimum(A[:, None, 2:], B[None, :, 2:])
    inter = (rb - lt).clamp_min(0).prod(-1)
    union = (a[:, 2] * a[:, 3])[:, None].float() + (b[:, 2] * b[:, 3])[None, :].float() - inter
    return torch.where(union > 0, inter / union.clamp_min(1e-30), torch.zeros_like(inter))


def nms_tensor(boxes: torch.Tensor, scores: torch.Tensor, classes: torch.Tensor, iou_threshold: float) -> torch.Tensor:
    """``nms`` on tensors: indices of the kept boxes (descending score). The IoU matrix is computed once
    on the device; the greedy pass walks it on the host."""
    order = torch.argsort(scores, descending=True, stable=True)
    m = box_iou_matrix(boxes[order], boxes[order]).cpu()
    same = (classes[order][:, None] == classes[order][None, :]).cpu()
    n = order.numel()
    keep, sup = [], torch.zeros(n, dtype=torch.bool)
    for i in range(n):
        if sup[i]:
            continue
        keep.append(i)
        sup |= (m[i] > iou_threshold) & same[i]  # later boxes it overlaps; earlier ones are decided
    return order[torch.tensor(keep, dtype=torch.long, device=order.device)]


class DetectionHead(Module):
    """Per-query box regression (sigmoid -> normalised cx, cy, w, h) and classification over the classes
    plus a background class (the last one)."""

    def __init__(self, embed_dim: int, num_classes: int, num_queries: int, device=None, dtype=torch.float32,
                 seed: int = 0):
        super().__init__()
        if embed_dim <= 0 or num_classes <= 0 or num_queries <= 0:
            raise ValueError("DetectionHead: all dims must be > 0")
        self.embed_dim, self.num_classes, self.num_queries = embed_dim, num_classes, num_queries
        g = torch.Generator().manual_seed(seed)
        self.box = Linear(embed_dim, 4, True, device, dtype)
        self.cls = Linear(embed_dim, num_classes + 1, True, device, dtype)
        with torch.no_grad():
            for lin in (self.box, self.cls):  # Xavier-uniform weights, zero biases
                lim = math.sqrt(6.0 / (lin.weight.shape[0] + lin.weight.shape[1]))
                lin.weight.copy_((torch.rand(lin.weight.shape, generator=g) * 2 - 1) * lim)
                lin.bias.zero_()

    def forward(self, queries: torch.Tensor):
        """queries [B, num_queries, D] -> (boxes [B, Q, 4] in (0, 1), class logits [B, Q, C + 1])."""
        if queries.shape[-2:] != (self.num_queries, self.embed_dim):
            raise ValueError("DetectionHead: queries shape mismatch")
        return torch.sigmoid(self.box(queries).float()), self.cls(queries).float()

    @torch.no_grad()
    def decode_boxes(self, boxes: torch.Tensor, cls_logits: torch.Tensor, score_threshold: float) -> list[list[Bbox]]:
        """Best foreground class per query (softmax over all classes, background excluded from the
        choice); queries whose best probability reaches the threshold become boxes."""
        probs = torch.softmax(cls_logits.double(), -1)[..., : self.num_classes]
        score, cls = probs.max(-1)
        out = []
        for b in range(boxes.shape[0]):
            row = []
            for q in range(boxes.shape[1]):
                if float(score[b, q]) >= score_threshold:
                    cx, cy, w, h = (float(x) for x in boxes[b, q])
                    row.append(Bbox(cx, cy, w, h, float(score[b, q]), int(cls[b, q])))
            out.append(row)
        return out

    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())


def mean_average_precision(predictions: list[list[Bbox]], ground_truth: list[list[Bbox]], iou_threshold: float,
                           num_classes: int) -> float:
    """Mean over classes of the area under the precision-recall curve (predictions in their given order,
    each matched greedily to the unmatched ground-truth box of best IoU); classes without ground truth
    count as zero, as in the reference."""
    if len(predictions) != len(ground_truth) or not predictions:
        return 0.0
    total = 0.0
    for c in range(num_classes):
        tp, n_gt = [], 0
        for preds, gts in zip(predictions, ground_truth):
            cg = [g for g in gts if g.class_id == c]
            n_gt += len(cg)
            matched = [False] * len(cg)
            for p in (p for p in preds if p.class_id == c):
                best, bi = -1.0, -1
                for i, g in enumerate(cg):
                    if not matched[i]:
                        v = iou(p, g)
                        if v > best:
                            best, bi = v, i
                if bi >= 0 and best >= iou_threshold:
                    matched[bi] = True
                    tp.append(1.0)
                else:
                    tp.append(0.0)
        if n_gt == 0:
            continue
        ctp = cfp = 0.0
        curve = [(1.0, 0.0)]
        for t in tp:
            ctp += t
            cfp += 1.0 - t
            curve.append((ctp / max(ctp + cfp, 1e-10), ctp / n_gt))
        curve.append((0.0, 1.0))
        total += sum((curve[i + 1][1] - curve[i][1]) * curve[i + 1][0] for i in range(len(curve) - 1))
    return total / num_classes if num_classes > 0 else 0.0


# --------------------------------------------------------------------------- segmentation
class SegDecoder(Module):
    """Per-patch linear classifier over patch tokens [B, N, D] -> logits [B, N, num_classes]."""

    def __init__(self, embed_dim: int, num_classes: int, device=None, dtype=torch.float32, seed: int = 0):
        super().__init__()
        if embed_dim <= 0 or num_classes <= 0:
            raise ValueError("SegDecoder: dims must be > 0")
        self.embed_dim, self.num_classes = embed_dim, num_classes
        self.proj = Linear(embed_dim, num_classes, True, device, dtype)
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            lim = math.sqrt(6.0 / (embed_dim + num_classes))
            self.proj.weight.copy_((torch.rand(self.proj.weight.shape, generator=g) * 2 - 1) * lim)
            self.proj.bias.zero_()

    def forward(self, patch_tokens: torch.Tensor) -> torch.Tensor:
        if patch_tokens.shape[-1] != self.embed_dim:
            raise ValueError("SegDecoder: tokens shape mismatch")
        return self.proj(patch_tokens)

    @staticmethod
    def predict_class(logits: torch.Tensor) -> torch.Tensor:
        return logits.argmax(-1)

    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())


class UpscaleDecoder(Module):
    """``SegDecoder`` on a grid_size x grid_size patch grid; ``upsample`` resamples the logits bilinearly to
    out_h x out_w pixels."""

    def __init__(self, embed_dim: int, num_classes: int, grid_size: int, out_h: int, out_w: int, device=None,
                 dtype=torch.float32, seed: int = 0):
        super().__init__()
        self.linear_dec = SegDecoder(embed_dim, num_classes, device, dtype, seed)
        self.grid_size, self.out_h, self.out_w = grid_size, out_h, out_w

    def forward(self, patch_tokens: torch.Tensor) -> torch.Tensor:
        if patch_tokens.shape[-2] != self.grid_size ** 2:
            raise ValueError("UpscaleDecoder: expected grid_size^2 patch tokens")
        return self.linear_dec(patch_tokens)

    def upsample(self, logits: torch.Tensor) -> torch.Tensor:
        """[B, G*G, C] -> [B, C, out_h, out_w]."""
        B, N, C = logits.shape
        g = logits.transpose(1, 2).reshape(B, C, self.grid_size, self.grid_size).float()
        return torch.nn.functional.interpolate(g, size=(self.out_h, self.out_w), mode="bilinear", align_corners=False)

    def num_params(self) -> int:
        return self.linear_dec.num_params()


def _flat(x):
    return torch.as_tensor(x).reshape(-1).long()


def per_class_iou(preds, gts, num_classes: int):
    """(IoU per class (nan where a class never occurs), mean over the classes that occur)."""
    p, g = _flat(preds), _flat(gts)
    if p.numel() != g.numel():
        raise ValueError("per_class_iou: length mismatch")
    ok = (p < num_classes) & (g < num_classes)
    p, g = p[ok], g[ok]
    tp = torch.bincount(p[p == g], minlength=num_classes).double()
    fp = torch.bincount(p[p != g], minlength=num_classes).double()
    fn = torch.bincount(g[p != g], minlength=num_classes).double()
    den = tp + fp + fn
    ious = torch.where(den > 0, tp / den.clamp_min(1), torch.full_like(den, float("nan")))
    valid = ious[~torch.isnan(ious)]
    return ious.tolist(), float(valid.mean()) if valid.numel() else 0.0


def pixel_accuracy(preds, gts) -> float:
    p, g = _flat(preds), _flat(gts)
    if p.numel() != g.numel():
        raise ValueError("pixel_accuracy: length mismatch")
    return float((p == g).double().mean()) if p.numel() else 0.0


def confusion_matrix(preds, gts, num_classes: int) -> torch.Tensor:
    """[num_classes, num_classes] counts, rows = ground truth, columns = prediction."""
    p, g = _flat(preds), _flat(gts)
    if p.numel() != g.numel():
        raise ValueError("confusion_matrix: length mismatch")
    ok = (p < num_classes) & (g < num_classes)
    return torch.bincount(g[ok] * num_classes + p[ok], minlength=num_classes ** 2).view(num_classes, num_classes)


def dice_coefficient(pred, gt) -> float:
    p, g = torch.as_tensor(pred).reshape(-1).bool(), torch.as_tensor(gt).reshape(-1).bool()
    if p.numel() != g.numel():
        raise ValueError("dice_coefficient: length mismatch")
    s = float(p.sum() + g.sum())
    return 1.0 if s < 1e-10 else 2.0 * float((p & g).sum()) / s


def seg_iou_pair(pred_mask, gt_mask) -> float:
    p, g = torch.as_tensor(pred_mask).reshape(-1).bool(), torch.as_tensor(gt_mask).reshape(-1).bool()
    if p.numel() != g.numel():
        raise ValueError("seg_iou_pair: length mismatch")
    union = float((p | g).sum())
    return 1.0 if union == 0 else float((p & g).sum()) / union


# --------------------------------------------------------------------------- backbones
class BackboneSize(enum.Enum):
    Tiny = "tiny"
    Small = "small"
    Base = "base"
    Large = "large"

    def config(self) -> ViTConfig:
        d, depth, heads = {"tiny": (192, 12, 3), "small": (384, 12, 6), "base": (768, 12, 12),
                           "large": (1024, 24, 16)}[self.value]
        return ViTConfig(hidden_dim=d, num_layers=depth, num_heads=heads, mlp_dim=4 * d)

    def embed_dim(self) -> int:
        return self.config().hidden_dim

    def depth(self) -> int:
        return self.config().num_layers


@dataclass
class BackboneConfig:
    size: BackboneSize = BackboneSize.Base
    use_cls_token: bool = True
    return_intermediate: bool = False
    return_blocks: list = field(default_factory=list)


class VitBackbone(Module):
    """A ViT without its classification head: token features for downstream heads."""

    def __init__(self, vit_cfg: ViTConfig, backbone_config: BackboneConfig | None = None, device=None,
                 dtype=torch.float32, seed: int = 0):
        super().__init__()
        self.vit = ViT(vit_cfg, device=device, dtype=dtype, seed=seed)
        self.backbone_config = backbone_config or BackboneConfig()

    @staticmethod
    def from_size(size: BackboneSize, device=None, dtype=torch.float32, seed: int = 0) -> "VitBackbone":
        return VitBackbone(size.config(), BackboneConfig(size=size), device, dtype, seed)

    def extract_features(self, images: torch.Tensor):
        """[B, C, H, W] -> final-norm token features [B, 1 + N, D]; with ``return_intermediate`` also the
        hidden states after the blocks listed in ``return_blocks``."""
        v = self.vit
        x = v.patch(v.patchify(images).to(v.patch.weight.dtype))
        x = torch.cat([v.cls_token.expand(x.shape[0], -1, -1), x], 1) + v.pos
        inter = []
        want = set(self.backbone_config.return_blocks)
        for i, layer in enumerate(v.encoder.layers):
            x = layer(x)
            if i in want:
                inter.append(x)
        h = v.encoder.final(x) if v.encoder.final is not None else x
        return (h, inter) if self.backbone_config.return_intermediate else h

    def _final(self, images):
        f = self.extract_features(images)
        return f[0] if isinstance(f, tuple) else f

    def extract_cls(self, images: torch.Tensor) -> torch.Tensor:
        return self._final(images)[:, 0]

    def extract_patches(self, images: torch.Tensor) -> torch.Tensor:
        return self._final(images)[:, 1:]

    def embed_dim(self) -> int:
        return self.vit.config.hidden_dim

    def total_params(self) -> int:
        return sum(p.numel() for p in self.parameters())


def micro_backbone(seed: int = 0, device=None, dtype=torch.float32) -> VitBackbone:
    """An 8x8 single-channel image, 4x4 patches, width 16, 2 heads, 2 blocks: for tests."""
    cfg = ViTConfig(image_size=8, patch_size=4, in_channels=1, hidden_dim=16, num_layers=2, num_heads=2, mlp_dim=32,
                    num_classes=2)
    return VitBackbone(cfg, BackboneConfig(size=BackboneSize.Tiny), device, dtype, seed)
