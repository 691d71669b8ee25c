"""Federated learning on the framework's tensors and collectives.

Reference: crates/brain-federated. Aggregation rules (server/aggregate.rs:10-100): FedAvg weighted by
client sample counts, FedProx (same server rule, proximal term on the client), coordinate-wise
trimmed mean and median. Secure aggregation (privacy/secure_agg.rs:9-80): every pair of clients
(i < j) shares a seeded mask that i adds and j subtracts, so the masks cancel in the sum. Differential
privacy (privacy/dp.rs:10-70): L2 clipping and Gaussian noise with
sigma = sensitivity * sqrt(2 ln(1.25 / delta)) / epsilon. Update compression
(compression/quantize.rs:21-60, compression/sparsify.rs:21): uniform min/max quantisation and top-k
sparsification. Client training (client/trainer.rs:15) and rounds (server/round.rs:10).

Design: client updates are lists of torch tensors (any device). In-process aggregation works on
stacked tensors (one vectorised sort per layer for the robust rules instead of a per-coordinate
loop). ``fed_avg_across_ranks`` runs one FedAvg round where every rank of a process group is a client:
one all-reduce of the sample-weighted update, so a GPU job aggregates over NVLink through the
framework's collectives. Masks and noise come from seeded torch generators, not the reference's LCG;
only the cancellation and noise-scale properties are kept.
"""
from __future__ import annotations

import enum
import math
from dataclasses import dataclass, field

import torch


class AggregationAlgorithm(enum.Enum):
    FED_AVG = "fedavg"
    FED_PROX = "fedprox"
    TRIMMED_MEAN = "trimmed_mean"
    MEDIAN = "median"


@dataclass
class ModelDelta:
    """One client's update: per-layer tensors and the number of samples it trained on."""
    client_id: int
    weights: list[torch.Tensor]
    num_samples: int


def fed_avg_aggregate(deltas: list[ModelDelta]) -> list[torch.Tensor]:
    """Sample-weighted average per layer; with zero total samples the first client's weights."""
    if not deltas:
        return []
    total = sum(d.num_samples for d in deltas)
    if total == 0:
        return [w.clone() for w in deltas[0].weights]
    out = []
    for layer in range(len(deltas[0].weights)):
        acc = torch.zeros_like(deltas[0].weights[layer], dtype=torch.float64)
        for d in deltas:
            acc += d.weights[layer].to(torch.float64) * (d.num_samples / total)
        out.append(acc.to(deltas[0].weights[layer].dtype))
    return out


def _stacked(deltas: list[ModelDelta], layer: int) -> torch.Tensor:
    return torch.stack([d.weights[layer].to(torch.float64) for d in deltas])


def trimmed_mean_aggregate(deltas: list[ModelDelta], trim_fraction: float) -> list[torch.Tensor]:
    """Per coordinate: drop the k lowest and k highest client values (k = floor(n * clamp(f, 0, 0.45)))
    and average the rest. Two or fewer clients fall back to FedAvg."""
    if not deltas:
        return []
    n = len(deltas)
    if n <= 2:
        return fed_avg_aggregate(deltas)
    k = int(math.floor(n * min(max(trim_fraction, 0.0), 0.45)))
    out = []
    for layer in range(len(deltas[0].weights)):
        s = torch.sort(_stacked(deltas, layer), dim=0).values
        out.append(s[k:n - k].mean(dim=0).to(deltas[0].weights[layer].dtype))
    return out


def median_aggregate(deltas: list[ModelDelta]) -> list[torch.Tensor]:
    """Coordinate-wise median; an even client count averages the two middle values."""
    if not deltas:
        return []
    n = len(deltas)
    out = []
    for layer in range(len(deltas[0].weights)):
        s = torch.sort(_stacked(deltas, layer), dim=0).values
        med = s[n // 2] if n % 2 else 0.5 * (s[n // 2 - 1] + s[n // 2])
        out.append(med.to(deltas[0].weights[layer].dtype))
    return out


def aggregate(deltas: list[ModelDelta], algorithm: AggregationAlgorithm = AggregationAlgorithm.FED_AVG,
              trim_fraction: float = 0.1) -> list[torch.Tensor]:
    if algorithm in (AggregationAlgorithm.FED_AVG, AggregationAlgorithm.FED_PROX):
        return fed_avg_aggregate(deltas)
    if algorithm == AggregationAlgorithm.TRIMMED_MEAN:
        return trimmed_mean_aggregate(deltas, trim_fraction)
    return median_aggregate(deltas)


def fed_avg_across_ranks(weights: list[torch.Tensor], num_samples: int, group=None) -> list[torch.Tensor]:
    """FedAvg where each rank of ``group`` is one client: all-reduce of (n_i * w_i) and of n_i, then a
    division. Every rank returns the same aggregate. Works on Gloo (CPU) and NCCL (GPU) groups."""
    import torch.distributed as dist

    if not weights:
        return []
    dev = weights[0].device
    flat = torch.cat([w.reshape(-1).to(torch.float32) for w in weights])
    buf = torch.cat([flat * float(num_samples), torch.tensor([float(num_samples)], device=dev)])
    dist.all_reduce(buf, group=group)
    total = float(buf[-1])
    agg = buf[:-1] / total if total > 0 else flat
    out, off = [], 0
    for w in weights:
        out.append(agg[off:off + w.numel()].view_as(w).to(w.dtype))
        off += w.numel()
    return out


def proximal_term(weights: list[torch.Tensor], global_weights: list[torch.Tensor], mu: float) -> torch.Tensor:
    """FedProx client penalty (mu / 2) * ||w - w_global||^2, added to the client loss."""
    tot = sum(((w - g.detach()) ** 2).sum() for w, g in zip(weights, global_weights))
    return 0.5 * mu * tot


# ------------------------------------------------------------------ secure aggregation
def _pair_seed(seed: int, i: int, j: int) -> int:
    a, b = min(i, j), max(i, j)
    return (seed + a * 0x9E3779B97F4A7C15 + b * 0x517CC1B727220A95) & 0x7FFFFFFFFFFFFFFF


def generate_mask(shape, pair_seed: int, device=None, dtype=torch.float64) -> torch.Tensor:
    """Uniform(-1, 1) mask from a seeded generator (same seed -> same mask on every client)."""
    g = torch.Generator(device="cpu").manual_seed(pair_seed)
    return (torch.rand(tuple(shape), generator=g, dtype=torch.float64) * 2 - 1).to(device=device, dtype=dtype)


class SecureAggregator:
    """Zero-sum pairwise masks: client i adds M_ij for every j > i and subtracts M_ji for every j < i."""

    def __init__(self, num_clients: int):
        self.num_clients = num_clients

    def generate_client_pairwise_mask(self, client_id: int, shape, seed: int, device=None,
                                      dtype=torch.float64) -> torch.Tensor:
        total = torch.zeros(tuple(shape), dtype=torch.float64)
        for peer in range(self.num_clients):
            if peer == client_id:
                continue
            m = generate_mask(shape, _pair_seed(seed, client_id, peer))
            total = total + m if client_id < peer else total - m
        return total.to(device=device, dtype=dtype)

    def mask_update(self, client_id: int, weights: list[torch.Tensor], seed: int) -> list[torch.Tensor]:
        return [mask_tensor(w, self.generate_client_pairwise_mask(client_id, w.shape, seed + i, w.device, w.dtype))
                for i, w in enumerate(weights)]


def mask_tensor(t: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    return t + mask


def unmask_tensor(t: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    return t - mask


# ------------------------------------------------------------------ differential privacy
@dataclass
class DpConfig:
    epsilon: float = 1.0
    delta: float = 1e-5
    sensitivity: float = 1.0
    clip_norm: float = 1.0


@dataclass
class GaussianNoise:
    config: DpConfig = field(default_factory=DpConfig)

    def compute_sigma(self) -> float:
        c = self.config
        return c.sensitivity * math.sqrt(2.0 * math.log(1.25 / c.delta)) / c.epsilon

    def privatize(self, t: torch.Tensor, seed: int) -> torch.Tensor:
        return add_dp_noise(clip_by_norm(t, self.config.clip_norm), self.compute_sigma(), seed)


@dataclass
class LaplaceNoise:
    config: DpConfig = field(default_factory=DpConfig)

    def scale(self) -> float:
        return self.config.sensitivity / self.config.epsilon

    def privatize(self, t: torch.Tensor, seed: int) -> torch.Tensor:
        g = torch.Generator(device="cpu").manual_seed(seed)
        u = torch.rand(t.shape, generator=g, dtype=torch.float64) - 0.5
        noise = -self.scale() * torch.sign(u) * torch.log1p(-2 * u.abs())
        return t + noise.to(device=t.device, dtype=t.dtype)


def clip_by_norm(t: torch.Tensor, max_norm: float) -> torch.Tensor:
    norm = float(t.to(torch.float64).norm())
    return t.clone() if norm <= max_norm else t * (max_norm / norm)


def add_dp_noise(t: torch.Tensor, sigma: float, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    noise = torch.randn(t.shape, generator=g, dtype=torch.float64) * sigma
    return t + noise.to(device=t.device, dtype=t.dtype)


# ------------------------------------------------------------------ compression
def quantize_tensor(t: torch.Tensor, bits: int):
    """Uniform quantisation to [0, 2^bits - 1] over [min, max]: returns (codes int32, min, max)."""
    lo, hi = float(t.min()), float(t.max())
    levels = (1 << bits) - 1
    if hi - lo < 1e-12:
        return torch.zeros(t.shape, dtype=torch.int32, device=t.device), lo, hi
    q = torch.round((t.to(torch.float64) - lo) / (hi - lo) * levels).clamp(0, levels).to(torch.int32)
    return q, lo, hi


def dequantize_tensor(q: torch.Tensor, lo: float, hi: float, bits: int) -> torch.Tensor:
    levels = (1 << bits) - 1
    if hi - lo < 1e-12:
        return torch.full(q.shape, lo, dtype=torch.float64, device=q.device)
    return lo + q.to(torch.float64) / levels * (hi - lo)


def top_k_sparsify(t: torch.Tensor, keep_fraction: float) -> torch.Tensor:
    """Keep the ceil(n * keep_fraction) largest-magnitude entries, zero the rest."""
    n = t.numel()
    k = max(1, min(n, int(math.ceil(n * keep_fraction))))
    flat = t.reshape(-1)
    idx = flat.abs().topk(k).indices
    out = torch.zeros_like(flat)
    out[idx] = flat[idx]
    return out.view_as(t)


# ------------------------------------------------------------------ client / server rounds
@dataclass
class RoundStats:
    round_id: int
    num_participants: int
    mean_client_loss: float = 0.0
    update_norm: float = 0.0


class FederatedClient:
    """Local SGD on a copy of the global model (``client/trainer.rs``); returns a ``ModelDelta`` of the
    trained weights. ``mu > 0`` adds the FedProx proximal term."""

    def __init__(self, client_id: int, model_fn, data, loss_fn, lr: float = 0.1, local_epochs: int = 1,
                 mu: float = 0.0):
        self.client_id, self.model_fn, self.data, self.loss_fn = client_id, model_fn, data, loss_fn
        self.lr, self.local_epochs, self.mu = lr, local_epochs, mu

    def train(self, global_weights: list[torch.Tensor]) -> tuple[ModelDelta, float]:
        model = self.model_fn()
        with torch.no_grad():
            for p, w in zip(model.parameters(), global_weights):
                p.copy_(w)
        opt = torch.optim.SGD(model.parameters(), lr=self.lr)
        n, last = 0, 0.0
        for _ in range(self.local_epochs):
            for x, y in self.data:
                loss = self.loss_fn(model(x), y)
                if self.mu > 0:
                    loss = loss + proximal_term(list(model.parameters()), global_weights, self.mu)
                opt.zero_grad()
                loss.backward()
                opt.step()
                n += x.shape[0]
                last = float(loss.detach())
        weights = [p.detach().clone() for p in model.parameters()]
        return ModelDelta(self.client_id, weights, n // max(1, self.local_epochs)), last


class FederatedServer:
    """Runs rounds: broadcast the global weights, train every client, aggregate (``server/round.rs``)."""

    def __init__(self, global_weights: list[torch.Tensor], algorithm=AggregationAlgorithm.FED_AVG,
                 trim_fraction: float = 0.1, secure: bool = False, seed: int = 0):
        self.weights = [w.detach().clone() for w in global_weights]
        self.algorithm, self.trim_fraction, self.secure, self.seed = algorithm, trim_fraction, secure, seed
        self.history: list[RoundStats] = []

    def run_round(self, clients: list[FederatedClient]) -> RoundStats:
        rid = len(self.history)
        results = [c.train(self.weights) for c in clients]
        deltas = [r[0] for r in results]
        if self.secure:
            if self.algorithm not in (AggregationAlgorithm.FED_AVG, AggregationAlgorithm.FED_PROX):
                raise ValueError("secure aggregation only supports sums (FedAvg / FedProx)")
            # each client masks its sample-weighted update; the server only sees masked sums
            agg = SecureAggregator(len(deltas))
            total = sum(d.num_samples for d in deltas)
            masked = [agg.mask_update(i, [w.to(torch.float64) * (d.num_samples / total) for w in d.weights],
                                      self.seed + 7919 * rid) for i, d in enumerate(deltas)]
            new = [sum(m[layer] for m in masked).to(self.weights[layer].dtype) for layer in range(len(self.weights))]
        else:
            new = aggregate(deltas, self.algorithm, self.trim_fraction)
        norm = math.sqrt(sum(float(((a.double() - b.double()) ** 2).sum()) for a, b in zip(new, self.weights)))
        self.weights = new
        stats = RoundStats(rid, len(clients), sum(r[1] for r in results) / max(1, len(results)), norm)
        self.history.append(stats)
        return stats


# ------------------------------------------------------------------ analysis and client helpers
# crates/brain-federated/src: utils.rs (sample_clients, stddev), ops.rs (l2_norm_delta, scale_delta),
# transform.rs (polyak_average, normalize_weights), analyze.rs (cosine_similarity_deltas,
# communication_cost_bytes, estimate_heterogeneity), monitor/mod.rs (FedMonitor: latest_loss,
# has_converged), process.rs (cosine_lr), client/trainer.rs (LocalTrainer / SgdTrainer).

def sample_clients(num_clients: int, fraction: float, round_idx: int, seed: int = 0, min_clients: int = 1) -> list[int]:
    """A seeded, round-dependent subset of max(min_clients, round(fraction * N)) client ids, sorted."""
    k = max(min_clients, int(round(fraction * num_clients)))
    g = torch.Generator().manual_seed(seed * 1_000_003 + round_idx)
    return sorted(torch.randperm(num_clients, generator=g)[:k].tolist())


def _flat(delta) -> torch.Tensor:
    ts = delta.tensors if hasattr(delta, "tensors") else delta
    return torch.cat([t.reshape(-1).double() for t in ts])


def l2_norm_delta(delta) -> float:
    return float(_flat(delta).norm())


def scale_delta(delta, s: float) -> list[torch.Tensor]:
    ts = delta.tensors if hasattr(delta, "tensors") else delta
    return [t * s for t in ts]


def cosine_similarity_deltas(a, b) -> float:
    fa, fb = _flat(a), _flat(b)
    d = fa.norm() * fb.norm()
    return float(fa @ fb / d) if d > 0 else 0.0


def estimate_heterogeneity(deltas) -> float:
    """1 - mean pairwise cosine similarity of the client updates (0: identical directions)."""
    n = len(deltas)
    if n < 2:
        return 0.0
    sims = [cosine_similarity_deltas(deltas[i], deltas[j]) for i in range(n) for j in range(i + 1, n)]
    return 1.0 - sum(sims) / len(sims)


def communication_cost_bytes(num_params: int, num_clients: int, rounds: int, bytes_per_param: float = 4.0,
                             bidirectional: bool = True) -> int:
    return int(num_params * bytes_per_param * num_clients * rounds * (2 if bidirectional else 1))


def polyak_average(avg: list[torch.Tensor], new: list[torch.Tensor], beta: float = 0.99) -> list[torch.Tensor]:
    return [beta * a + (1 - beta) * n for a, n in zip(avg, new)]


def normalize_weights(weights) -> list[float]:
    s = float(sum(weights))
    return [float(w) / s for w in weights] if s > 0 else [1.0 / len(weights)] * len(weights)


def stddev(values) -> float:
    v = torch.as_tensor(list(values), dtype=torch.float64)
    return float(v.std(unbiased=False)) if v.numel() else 0.0


def cosine_lr(base_lr: float, round_idx: int, total_rounds: int, min_lr: float = 0.0) -> float:
    import math
    t = min(max(round_idx / max(total_rounds, 1), 0.0), 1.0)
    return min_lr + 0.5 * (base_lr - min_lr) * (1 + math.cos(math.pi * t))


class FedMonitor:
    """Per-round global losses; converged when the last ``window`` rounds improved by less than ``tol``."""

    def __init__(self, window: int = 3, tol: float = 1e-4):
        self.window, self.tol, self.losses = window, tol, []

    def record(self, loss: float) -> None:
        self.losses.append(float(loss))

    def latest_loss(self):
        return self.losses[-1] if self.losses else None

    def has_converged(self) -> bool:
        if len(self.losses) <= self.window:
            return False
        return self.losses[-self.window - 1] - min(self.losses[-self.window:]) < self.tol


class LocalTrainer:
    """Local SGD epochs of a client on its data: returns the parameter delta (new - old) and sample count."""

    def __init__(self, model, loss_fn, lr: float = 0.01, epochs: int = 1, weight_decay: float = 0.0):
        self.model, self.loss_fn, self.lr, self.epochs, self.wd = model, loss_fn, lr, epochs, weight_decay

    def train(self, batches):
        params = [p for p in self.model.parameters() if p.requires_grad]
        before = [p.detach().clone() for p in params]
        opt = torch.optim.SGD(params, lr=self.lr, weight_decay=self.wd)
        n = 0
        for _ in range(self.epochs):
            for x, y in batches:
                opt.zero_grad()
                self.loss_fn(self.model(x), y).backward()
                opt.step()
                n += x.shape[0]
        return [p.detach() - b for p, b in zip(params, before)], n // max(self.epochs, 1)


SgdTrainer = LocalTrainer
