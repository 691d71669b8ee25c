"""Evaluation metrics (crates/brain-metric/src/): classification, ranking, regression, NLP,
segmentation, detection, clustering, calibration, plus streaming aggregation (``track.rs``).
All take torch tensors (any device) and return Python floats."""
from __future__ import annotations

import math
from collections import Counter

import torch


def _f(x):
    return x.detach().float()


# ------------------------------------------------------------------ classification
def accuracy(pred_or_logits, target) -> float:
    p = pred_or_logits.argmax(-1) if pred_or_logits.dim() > target.dim() else pred_or_logits
    return float((p == target).float().mean())


def top_k_accuracy(logits, target, k=5) -> float:
    top = logits.topk(k, -1).indices
    return float((top == target[..., None]).any(-1).float().mean())


def confusion_matrix(pred, target, num_classes: int) -> torch.Tensor:
    idx = target.long() * num_classes + pred.long()
    return torch.bincount(idx.flatten(), minlength=num_classes * num_classes).view(num_classes, num_classes)


def precision_recall_f1(pred, target, num_classes: int, average: str = "macro"):
    cm = confusion_matrix(pred, target, num_classes).double()
    tp = cm.diag()
    fp = cm.sum(0) - tp
    fn = cm.sum(1) - tp
    if average == "micro":
        p = tp.sum() / (tp.sum() + fp.sum()).clamp_min(1)
        r = tp.sum() / (tp.sum() + fn.sum()).clamp_min(1)
        f = 2 * p * r / (p + r).clamp_min(1e-12)
        return float(p), float(r), float(f)
    p = tp / (tp + fp).clamp_min(1)
    r = tp / (tp + fn).clamp_min(1)
    f = 2 * p * r / (p + r).clamp_min(1e-12)
    if average == "weighted":
        w = cm.sum(1) / cm.sum()
        return float((p * w).sum()), float((r * w).sum()), float((f * w).sum())
    return float(p.mean()), float(r.mean()), float(f.mean())


def matthews_corrcoef(pred, target) -> float:
    p, t = pred.bool().double(), target.bool().double()
    tp = (p * t).sum()
    tn = ((1 - p) * (1 - t)).sum()
    fp = (p * (1 - t)).sum()
    fn = ((1 - p) * t).sum()
    den = math.sqrt(float((tp + fp) * (tp + fn) * (tn + fp) * (tn + fn))) or 1.0
    return float(tp * tn - fp * fn) / den


def cohen_kappa(pred, target, num_classes: int) -> float:
    cm = confusion_matrix(pred, target, num_classes).double()
    n = cm.sum()
    po = cm.diag().sum() / n
    pe = (cm.sum(0) * cm.sum(1)).sum() / (n * n)
    return float((po - pe) / (1 - pe)) if pe < 1 else 0.0


def roc_auc(scores, target) -> float:
    """Binary ROC-AUC by the rank statistic (ties averaged)."""
    s, t = _f(scores).flatten(), target.flatten().bool()
    order = s.argsort()
    ranks = torch.empty_like(s)
    ranks[order] = torch.arange(1, len(s) + 1, dtype=s.dtype, device=s.device)
    for v in s.unique():  # average ties
        m = s == v
        if m.sum() > 1:
            ranks[m] = ranks[m].mean()
    npos, nneg = int(t.sum()), int((~t).sum())
    if npos == 0 or nneg == 0:
        return float("nan")
    return float((ranks[t].sum() - npos * (npos + 1) / 2) / (npos * nneg))


def average_precision(scores, target) -> float:
    s, t = _f(scores).flatten(), target.flatten().float()
    order = s.argsort(descending=True)
    t = t[order]
    tp = t.cumsum(0)
    prec = tp / torch.arange(1, len(t) + 1, device=t.device)
    return float((prec * t).sum() / t.sum().clamp_min(1))


pr_auc = average_precision


def log_loss(probs, target, eps=1e-12) -> float:
    p = _f(probs).clamp(eps, 1 - eps)
    return float(-(target * p.log() + (1 - target) * (1 - p).log()).mean())


def expected_calibration_error(probs, target, n_bins=15) -> float:
    conf, pred = _f(probs).max(-1)
    acc = (pred == target).float()
    ece = 0.0
    edges = torch.linspace(0, 1, n_bins + 1)
    for lo, hi in zip(edges[:-1], edges[1:]):
        m = (conf > lo) & (conf <= hi)
        if m.any():
            ece += float(m.float().mean() * (conf[m].mean() - acc[m].mean()).abs())
    return ece


def brier_score(probs, target) -> float:
    oh = torch.nn.functional.one_hot(target, probs.shape[-1]).float()
    return float(((_f(probs) - oh) ** 2).sum(-1).mean())


def hamming_loss(pred, target) -> float:
    return float((pred != target).float().mean())


def multilabel_f1(pred, target) -> float:
    p, t = pred.bool(), target.bool()
    tp = (p & t).sum().double()
    return float(2 * tp / (p.sum() + t.sum()).clamp_min(1))


# ------------------------------------------------------------------ regression / time series
def mse(p, t) -> float:
    return float(((_f(p) - _f(t)) ** 2).mean())


def rmse(p, t) -> float:
    return math.sqrt(mse(p, t))


def mae(p, t) -> float:
    return float((_f(p) - _f(t)).abs().mean())


def mape(p, t, eps=1e-8) -> float:
    return float(((_f(p) - _f(t)).abs() / _f(t).abs().clamp_min(eps)).mean() * 100)


def smape(p, t, eps=1e-8) -> float:
    p, t = _f(p), _f(t)
    return float((2 * (p - t).abs() / (p.abs() + t.abs()).clamp_min(eps)).mean() * 100)


def r2_score(p, t) -> float:
    p, t = _f(p), _f(t)
    ss_res = ((t - p) ** 2).sum()
    ss_tot = ((t - t.mean()) ** 2).sum()
    return float(1 - ss_res / ss_tot.clamp_min(1e-12))


def explained_variance(p, t) -> float:
    p, t = _f(p), _f(t)
    return float(1 - (t - p).var() / t.var().clamp_min(1e-12))


def pearson(p, t) -> float:
    p, t = _f(p).flatten(), _f(t).flatten()
    pc, tc = p - p.mean(), t - t.mean()
    return float((pc * tc).sum() / (pc.norm() * tc.norm()).clamp_min(1e-12))


def spearman(p, t) -> float:
    return pearson(_f(p).flatten().argsort().argsort().float(), _f(t).flatten().argsort().argsort().float())


# ------------------------------------------------------------------ ranking
def ndcg_at_k(scores, relevance, k=10) -> float:
    order = _f(scores).argsort(descending=True)[:k]
    rel = _f(relevance)[order]
    disc = 1.0 / torch.log2(torch.arange(2, len(rel) + 2, dtype=torch.float32, device=rel.device))
    dcg = ((2 ** rel - 1) * disc).sum()
    ideal = _f(relevance).sort(descending=True).values[:k]
    idcg = ((2 ** ideal - 1) * disc[:len(ideal)]).sum()
    return float(dcg / idcg.clamp_min(1e-12))


def mean_reciprocal_rank(scores, relevant_index) -> float:
    ranks = (_f(scores) > _f(scores).gather(-1, relevant_index[..., None])).sum(-1) + 1
    return float((1.0 / ranks.float()).mean())


def precision_at_k(scores, relevance, k=10) -> float:
    order = _f(scores).argsort(descending=True)[:k]
    return float((_f(relevance)[order] > 0).float().mean())


def recall_at_k(scores, relevance, k=10) -> float:
    order = _f(scores).argsort(descending=True)[:k]
    return float((_f(relevance)[order] > 0).sum() / (_f(relevance) > 0).sum().clamp_min(1))


# ------------------------------------------------------------------ NLP
def perplexity(mean_nll: float) -> float:
    return math.exp(min(mean_nll, 700.0))


def _ngrams(toks, n):
    return Counter(tuple(toks[i:i + n]) for i in range(len(toks) - n + 1))


def bleu(candidate: list, references: list[list], max_n: int = 4, smooth: bool = True) -> float:
    """Corpus-style BLEU for one sentence (geometric mean of clipped n-gram precisions, brevity penalty)."""
    logs = []
    for n in range(1, max_n + 1):
        c = _ngrams(candidate, n)
        mx = Counter()
        for r in references:
            for g, k in _ngrams(r, n).items():
                mx[g] = max(mx[g], k)
        clipped = sum(min(k, mx[g]) for g, k in c.items())
        total = max(1, sum(c.values()))
        p = (clipped + (1 if smooth else 0)) / (total + (1 if smooth else 0))
        logs.append(math.log(p) if p > 0 else -math.inf)
    ref_len = min((abs(len(r) - len(candidate)), len(r)) for r in references)[1]
    bp = 1.0 if len(candidate) > ref_len else math.exp(1 - ref_len / max(1, len(candidate)))
    return bp * math.exp(sum(logs) / max_n)


def rouge_n(candidate: list, reference: list, n: int = 1) -> float:
    c, r = _ngrams(candidate, n), _ngrams(reference, n)
    overlap = sum(min(k, r[g]) for g, k in c.items())
    return overlap / max(1, sum(r.values()))


def rouge_l(candidate: list, reference: list) -> float:
    m, n = len(candidate), len(reference)
    dp = [[0] * (n + 1) for _ in range(m + 1)]
    for i in range(m):
        for j in range(n):
            dp[i + 1][j + 1] = dp[i][j] + 1 if candidate[i] == reference[j] else max(dp[i][j + 1], dp[i + 1][j])
    lcs = dp[m][n]
    if lcs == 0:
        return 0.0
    p, r = lcs / m, lcs / n
    return 2 * p * r / (p + r)


def word_error_rate(hyp: list, ref: list) -> float:
    d = list(range(len(ref) + 1))
    for i, h in enumerate(hyp, 1):
        prev, d[0] = d[0], i
        for j, r in enumerate(ref, 1):
            cur = min(d[j] + 1, d[j - 1] + 1, prev + (h != r))
            prev, d[j] = d[j], cur
    return d[len(ref)] / max(1, len(ref))


# ------------------------------------------------------------------ segmentation / detection
def iou(pred_mask, target_mask) -> float:
    p, t = pred_mask.bool(), target_mask.bool()
    return float((p & t).sum() / (p | t).sum().clamp_min(1))


def dice_coefficient(pred_mask, target_mask) -> float:
    p, t = pred_mask.bool(), target_mask.bool()
    return float(2 * (p & t).sum() / (p.sum() + t.sum()).clamp_min(1))


def mean_iou(pred, target, num_classes: int) -> float:
    cm = confusion_matrix(pred.flatten(), target.flatten(), num_classes).double()
    inter = cm.diag()
    union = cm.sum(0) + cm.sum(1) - inter
    valid = union > 0
    return float((inter[valid] / union[valid]).mean())


def box_iou(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Pairwise IoU of [N,4] and [M,4] boxes (x1, y1, x2, y2)."""
    area = lambda x: (x[:, 2] - x[:, 0]).clamp_min(0) * (x[:, 3] - x[:, 1]).clamp_min(0)  # noqa: E731
    lt = torch.maximum(a[:, None, :2], b[None, :, :2])
    rb = torch.minimum(a[:, None, 2:], b[None, :, 2:])
    wh = (rb - lt).clamp_min(0)
    inter = wh[..., 0] * wh[..., 1]
    return inter / (area(a)[:, None] + area(b)[None, :] - inter).clamp_min(1e-12)


def average_precision_detection(pred_boxes, scores, gt_boxes, iou_thresh=0.5) -> float:
    order = scores.argsort(descending=True)
    matched = torch.zeros(len(gt_boxes), dtype=torch.bool)
    tps = []
    for i in order.tolist():
        if len(gt_boxes) == 0:
            tps.append(0)
            continue
        ious = box_iou(pred_boxes[i:i + 1].float(), gt_boxes.float())[0]
        j = int(ious.argmax())
        if ious[j] >= iou_thresh and not matched[j]:
            matched[j] = True
            tps.append(1)
        else:
            tps.append(0)
    if not tps:
        return 0.0
    return average_precision(torch.arange(len(tps), 0, -1).float(), torch.tensor(tps)) * sum(tps) / max(1, len(gt_boxes))


# ------------------------------------------------------------------ clustering
def silhouette_score(x: torch.Tensor, labels: torch.Tensor) -> float:
    d = torch.cdist(_f(x), _f(x))
    s = []
    for i in range(len(x)):
        same = labels == labels[i]
        a = d[i][same].sum() / max(1, int(same.sum()) - 1)
        others = [d[i][labels == c].mean() for c in labels.unique() if c != labels[i]]
        b = min(others) if others else torch.tensor(0.0)
        s.append(float((b - a) / max(float(a), float(b), 1e-12)))
    return sum(s) / len(s)


def adjusted_rand_index(a: torch.Tensor, b: torch.Tensor) -> float:
    from math import comb
    ua, ub = a.unique(), b.unique()
    cont = torch.stack([torch.stack([((a == i) & (b == j)).sum() for j in ub]) for i in ua]).long()
    s_ij = sum(comb(int(v), 2) for v in cont.flatten())
    s_a = sum(comb(int(v), 2) for v in cont.sum(1))
    s_b = sum(comb(int(v), 2) for v in cont.sum(0))
    n = comb(len(a), 2)
    exp = s_a * s_b / n if n else 0
    mx = (s_a + s_b) / 2
    return (s_ij - exp) / (mx - exp) if mx != exp else 1.0


# ------------------------------------------------------------------ streaming
class MetricTracker:
    """Streaming mean/min/max/count of named scalars (track.rs / aggregate.rs)."""

    def __init__(self):
        self.data: dict[str, list[float]] = {}

    def update(self, **kv):
        for k, v in kv.items():
            self.data.setdefault(k, []).append(float(v))

    def mean(self, k) -> float:
        v = self.data.get(k, [])
        return sum(v) / len(v) if v else float("nan")

    def summary(self) -> dict:
        return {k: {"mean": sum(v) / len(v), "min": min(v), "max": max(v), "count": len(v)}
                for k, v in self.data.items() if v}

    def report(self) -> str:
        return "\n".join(f"{k}: mean={s['mean']:.6g} min={s['min']:.6g} max={s['max']:.6g} n={s['count']}"
                         for k, s in self.summary().items())
