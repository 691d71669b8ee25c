"""Evaluation metrics (crates/brain-metric/src/): classification, ranking, regression, NLP,
segmentation, detection, clustering, calibration, plus streaming aggregation (``track.rs``).
All take torch tensors (any device) and return Python floats."""
from __future__ import annotations

import math
from collections import Counter
from dataclasses import dataclass, field

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
    """Streaming count-weighted mean and min/max of named scalars (track.rs / aggregate.rs):
    ``update(loss=0.3, acc=0.9)`` adds one sample per name; ``update("loss", 0.3, count=32)`` adds a
    batch-mean weighted by its sample count (the reference's form)."""

    def __init__(self):
        self.sums: dict[str, float] = {}
        self.counts: dict[str, int] = {}
        self.mins: dict[str, float] = {}
        self.maxs: dict[str, float] = {}

    def update(self, name: str | None = None, value: float | None = None, count: int = 1, **kv):
        items = dict(kv)
        if name is not None:
            items[name] = value
        for k, v in items.items():
            v = float(v)
            self.sums[k] = self.sums.get(k, 0.0) + v * count
            self.counts[k] = self.counts.get(k, 0) + count
            self.mins[k] = min(self.mins.get(k, v), v)
            self.maxs[k] = max(self.maxs.get(k, v), v)

    def mean(self, k) -> float:
        c = self.counts.get(k, 0)
        return self.sums[k] / c if c else float("nan")

    def summary(self) -> dict:
        return {k: {"mean": self.sums[k] / c, "min": self.mins[k], "max": self.maxs[k], "count": c}
                for k, c in self.counts.items() if c}

    def report(self) -> str:
        return "\n".join(f"{k}: mean={s['mean']:.6g} min={s['min']:.6g} max={s['max']:.6g} n={s['count']}"
                         for k, s in self.summary().items())

    def reset(self) -> None:
        for d in (self.sums, self.counts, self.mins, self.maxs):
            d.clear()


# ------------------------------------------------------------------ reports, calibration, imbalance, time series
def g_mean_score(tp: int, tn: int, fp: int, fn: int) -> float:
    """sqrt(sensitivity x specificity), each 0 when its denominator is 0
    (crates/brain-metric/src/imbalance.rs)."""
    sens = tp / (tp + fn) if tp + fn else 0.0
    spec = tn / (tn + fp) if tn + fp else 0.0
    return math.sqrt(sens * spec)


def mase_score(forecast, actual, seasonality_lag: int = 1) -> float:
    """MAE of the forecast over the MAE of the seasonal-naive forecast y[t - lag] (1 when that is 0; 0 for
    series no longer than the lag; crates/brain-metric/src/time_series.rs)."""
    f, y = _f(forecast).reshape(-1), _f(actual).reshape(-1)
    n = min(f.numel(), y.numel())
    if n <= seasonality_lag:
        return 0.0
    mae_f = float((f[:n] - y[:n]).abs().mean())
    mae_n = float((y[seasonality_lag:n] - y[:n - seasonality_lag]).abs().mean())
    return mae_f / mae_n if mae_n > 0 else 1.0


def forecast_bias(forecast, actual) -> float:
    f, y = _f(forecast).reshape(-1), _f(actual).reshape(-1)
    n = min(f.numel(), y.numel())
    return float((f[:n] - y[:n]).mean()) if n else 0.0


def median_absolute_error(p, t) -> float:
    return float((_f(p) - _f(t)).abs().median())


def huber_metric(p, t, delta: float = 1.0) -> float:
    r = (_f(p) - _f(t)).abs()
    return float(torch.where(r <= delta, 0.5 * r * r, delta * (r - 0.5 * delta)).mean())


def meteor_score_lite(hypothesis, reference) -> float:
    """Unigram-set matches m: P = m / |hyp|, R = m / |ref|, score 10 P R / (R + 9 P) (0 without matches)."""
    m = len(set(hypothesis) & set(reference))
    if m == 0:
        return 0.0
    p, r = m / max(len(hypothesis), 1), m / max(len(reference), 1)
    return 10 * p * r / (r + 9 * p)


def cluster_purity(assignments, labels) -> float:
    """Fraction of points that carry their cluster's majority label."""
    a, y = torch.as_tensor(assignments).long().reshape(-1), torch.as_tensor(labels).long().reshape(-1)
    n = min(a.numel(), y.numel())
    if n == 0:
        return 0.0
    a, y = a[:n], y[:n]
    ny = int(y.max()) + 1
    counts = torch.zeros(int(a.max()) + 1, ny, dtype=torch.long).index_put_((a, y), torch.ones(n, dtype=torch.long),
                                                                           accumulate=True)
    return float(counts.max(1).values.sum()) / n


def threshold_sweep_roc(probs, targets, num_thresholds: int = 100):
    """(TPR, FPR) at thresholds k / num_thresholds, k = 0..num_thresholds (predict positive when p >= t),
    all thresholds at once as one [T, N] comparison."""
    p, y = _f(probs).reshape(-1), torch.as_tensor(targets).reshape(-1) == 1
    th = torch.arange(num_thresholds + 1, dtype=p.dtype) / num_thresholds
    pred = p[None, :] >= th[:, None]
    npos, nneg = int(y.sum()), int((~y).sum())
    tpr = (pred & y).sum(1).double() / npos if npos else torch.zeros(len(th), dtype=torch.float64)
    fpr = (pred & ~y).sum(1).double() / nneg if nneg else torch.zeros(len(th), dtype=torch.float64)
    return tpr, fpr


def pr_auc_score(scores, target) -> float:
    """Area under the precision-recall curve by the trapezoid rule over the sorted scores."""
    s, y = _f(scores).reshape(-1), torch.as_tensor(target).reshape(-1).double()
    order = torch.argsort(s, descending=True, stable=True)
    y = y[order]
    tp = torch.cumsum(y, 0)
    prec = tp / torch.arange(1, len(y) + 1, dtype=torch.float64)
    rec = tp / y.sum().clamp_min(1)
    rec = torch.cat([torch.zeros(1, dtype=torch.float64), rec])
    prec = torch.cat([prec[:1], prec])
    return float(torch.trapz(prec, rec))


def multiclass_roc_auc(probs, target) -> float:
    """Macro one-vs-rest ROC AUC over the classes present in ``target``."""
    pr = _f(probs)
    t = torch.as_tensor(target).long().reshape(-1)
    aucs = [roc_auc(pr[:, c], (t == c).long()) for c in range(pr.shape[1]) if bool((t == c).any()) and bool((t != c).any())]
    return float(sum(aucs) / len(aucs)) if aucs else 0.0


@dataclass
class CalibrationReport:
    ece: float = 0.0
    mce: float = 0.0
    bin_accuracies: list = field(default_factory=list)
    bin_confidences: list = field(default_factory=list)


def compute_calibration(confidences, correct, num_bins: int = 15) -> CalibrationReport:
    """Expected and maximum calibration error over uniform confidence bins (confidence clamped below 1)."""
    c = _f(confidences).reshape(-1).clamp(0.0, 1.0 - 1e-9)
    ok = torch.as_tensor(correct).reshape(-1).double()
    b = (c * num_bins).floor().long().clamp(max=num_bins - 1)
    cnt = torch.bincount(b, minlength=num_bins).double()
    acc = torch.bincount(b, ok, minlength=num_bins) / cnt.clamp_min(1)
    conf = torch.bincount(b, c, minlength=num_bins) / cnt.clamp_min(1)
    gap = (acc - conf).abs() * (cnt > 0)
    n = c.numel()
    return CalibrationReport(float((cnt / max(n, 1) * gap).sum()), float(gap.max()) if n else 0.0, acc.tolist(),
                             conf.tolist())


@dataclass
class AggregateReport:
    mean: float = 0.0
    std_dev: float = 0.0
    min: float = 0.0
    max: float = 0.0
    ci_95_lower: float = 0.0
    ci_95_upper: float = 0.0


def aggregate_metric_runs(values) -> AggregateReport:
    """Mean, sample standard deviation and a normal 95 % interval mean +- 1.96 sd / sqrt(n) over runs."""
    v = torch.as_tensor(list(values), dtype=torch.float64)
    n = v.numel()
    if n == 0:
        return AggregateReport()
    sd = float(v.std()) if n > 1 else 0.0
    mg = 1.96 * sd / math.sqrt(n) if n > 1 else 0.0
    m = float(v.mean())
    return AggregateReport(m, sd, float(v.min()), float(v.max()), m - mg, m + mg)


@dataclass
class CompareReport:
    delta: float
    relative_gain_pct: float
    is_model_a_better: bool


def compare_models(score_a: float, score_b: float) -> CompareReport:
    d = score_a - score_b
    return CompareReport(d, d / score_b * 100.0 if abs(score_b) > 1e-12 else 0.0, d > 0)


def format_markdown_report(metrics: dict, title: str = "Metrics") -> str:
    rows = "\n".join(f"| {k} | {v:.4f} |" for k, v in sorted(metrics.items()))
    return f"## {title}\n\n| metric | value |\n|---|---|\n{rows}\n"


def format_csv_report(metrics: dict) -> str:
    return "metric,value\n" + "".join(f"{k},{v}\n" for k, v in sorted(metrics.items()))


# ------------------------------------------------------------------ the reference's spellings and helpers
# crates/brain-metric/src: classification/mod.rs (accuracy_score), classification/auc.rs (roc_auc_score),
# imbalance.rs (matthews_correlation_coefficient), regression/mod.rs (mse/rmse/mae/mape_score),
# stats/mod.rs (pearson_correlation), nlp (sentence_bleu, perplexity_score, edit_distance_levenshtein),
# multilabel.rs (exact_match_ratio), segmentation/mod.rs (miou_and_pixel_accuracy), detection (bbox_iou),
# ops.rs (logits_to_predictions, binarize_probs), utils.rs (topk_indices, stable_divide, bin_values_uniform).
accuracy_score = accuracy
roc_auc_score = roc_auc
matthews_correlation_coefficient = matthews_corrcoef
mse_score = mse
rmse_score = rmse
mae_score = mae
mape_score = mape
pearson_correlation = pearson
perplexity_score = perplexity
bbox_iou = box_iou


def sentence_bleu(candidate, references, max_n: int = 4, smooth: bool = True) -> float:
    return bleu(candidate, references, max_n, smooth)


def edit_distance_levenshtein(a, b) -> int:
    from .text_ops import levenshtein_distance
    return levenshtein_distance(a, b)


def exact_match_ratio(pred: torch.Tensor, target: torch.Tensor) -> float:
    """Share of samples whose whole label vector matches (multi-label subset accuracy)."""
    return float((pred.bool() == target.bool()).all(-1).float().mean())


def miou_and_pixel_accuracy(pred: torch.Tensor, target: torch.Tensor, num_classes: int):
    """(mean IoU over classes present in either map, pixel accuracy) of integer label maps."""
    p, t = pred.reshape(-1).long(), target.reshape(-1).long()
    cm = torch.bincount(t * num_classes + p, minlength=num_classes * num_classes).reshape(num_classes, num_classes)
    inter = cm.diag().double()
    union = cm.sum(0).double() + cm.sum(1).double() - inter
    present = union > 0
    miou = float((inter[present] / union[present]).mean()) if present.any() else 0.0
    return miou, float(inter.sum() / cm.sum().clamp_min(1))


def logits_to_predictions(logits: torch.Tensor) -> torch.Tensor:
    return logits.argmax(-1)


def binarize_probs(probs: torch.Tensor, threshold: float = 0.5) -> torch.Tensor:
    return (probs >= threshold).long()


def topk_indices(values: torch.Tensor, k: int) -> torch.Tensor:
    return torch.topk(values, min(k, values.shape[-1]), dim=-1).indices


def stable_divide(num: float, den: float, default: float = 0.0) -> float:
    return num / den if den != 0 else default


def bin_values_uniform(values: torch.Tensor, num_bins: int, lo: float = 0.0, hi: float = 1.0) -> torch.Tensor:
    """Bin index in [0, num_bins) of each value over the uniform partition of [lo, hi] (edges clamp)."""
    idx = ((values - lo) / (hi - lo) * num_bins).floor().long()
    return idx.clamp(0, num_bins - 1)


_METRICS = {"accuracy": accuracy, "mse": mse, "rmse": rmse, "mae": mae, "mape": mape, "r2": r2_score,
            "pearson": pearson, "spearman": spearman, "roc_auc": roc_auc, "mcc": matthews_corrcoef}


def metric_names() -> list[str]:
    return sorted(_METRICS)


def compute_metric(kind: str, pred, target, **kw):
    if kind not in _METRICS:
        raise ValueError(f"unknown metric {kind!r}; known: {', '.join(metric_names())}")
    return _METRICS[kind](pred, target, **kw)
