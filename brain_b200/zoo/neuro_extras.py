"""Neuroevolution building blocks on populations as tensors: benchmark functions, crossover operators,
ranking and statistics, termination, the reference's xorshift generator, and HyperNEAT (a CPPN queried
over a 2-D substrate to produce a weight matrix in one batched evaluation).

Reference: crates/brain-neuroevolution/src/benchmark.rs (sphere, Rosenbrock, Rastrigin, Ackley),
crossover.rs (single-point, uniform, BLX-alpha, SBX), utils.rs (FastRng, rank_fitness), fitness.rs
(FitnessStats), ga/termination.rs (TerminationConfig/Tracker), hyperneat/cppn.rs (Cppn, activations),
hyperneat/substrate.rs (SubstrateGrid2D, generate_weight_matrix), parallel.rs
(evaluate_population_parallel), checkpoint.rs (EvoCheckpoint).

A population is a [P, D] tensor on any device: a benchmark function evaluates all P genomes at once,
and a crossover produces [P, D] children from two [P, D] parent tensors with one draw tensor. The
reference's CPPN always returns gaussian(distance) - 0.5; ``Cppn`` here is an evolvable compositional
network (a DAG of nodes with the reference's activation set) whose default genome reproduces that
function exactly.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

_M64 = (1 << 64) - 1


# ------------------------------------------------------------------------------------------ generator
class FastRng:
    """xorshift64 (shifts 13, 7, 17; Marsaglia 2003) with the reference's seeding: seed 0 becomes
    0x853c49e6748fea9b. ``next_f64`` takes the top 53 bits."""

    def __init__(self, seed: int):
        self.state = (seed & _M64) or 0x853C49E6748FEA9B

    def next_u64(self) -> int:
        x = self.state
        x ^= (x << 13) & _M64
        x ^= x >> 7
        x ^= (x << 17) & _M64
        self.state = x
        return x

    def next_f64(self) -> float:
        return (self.next_u64() >> 11) / float(1 << 53)

    def sample_range(self, lo: float, hi: float) -> float:
        return lo + self.next_f64() * (hi - lo)

    def sample_gaussian(self, mean: float, std: float) -> float:
        u1 = max(self.next_f64(), 1e-15)
        u2 = self.next_f64()
        return mean + std * math.sqrt(-2.0 * math.log(u1)) * math.cos(2.0 * math.pi * u2)

    def uniform(self, n: int) -> torch.Tensor:
        return torch.tensor([self.next_f64() for _ in range(n)], dtype=torch.float64)


# ------------------------------------------------------------------------------------------ benchmarks
def sphere_fn(x: torch.Tensor) -> torch.Tensor:
    """sum x^2 over the last dimension ([P, D] -> [P])."""
    return (x * x).sum(-1)


def rosenbrock_fn(x: torch.Tensor) -> torch.Tensor:
    """sum 100 (x_{i+1} - x_i^2)^2 + (1 - x_i)^2 (0 for fewer than two dimensions)."""
    if x.shape[-1] < 2:
        return x.new_zeros(x.shape[:-1])
    a, b = x[..., :-1], x[..., 1:]
    return (100.0 * (b - a * a) ** 2 + (1.0 - a) ** 2).sum(-1)


def rastrigin_fn(x: torch.Tensor) -> torch.Tensor:
    return 10.0 * x.shape[-1] + (x * x - 10.0 * torch.cos(2.0 * math.pi * x)).sum(-1)


def ackley_fn(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1]
    if d == 0:
        return x.new_zeros(x.shape[:-1])
    t1 = -20.0 * torch.exp(-0.2 * torch.sqrt((x * x).mean(-1)))
    t2 = -torch.exp(torch.cos(2.0 * math.pi * x).mean(-1))
    return t1 + t2 + 20.0 + math.e


# ------------------------------------------------------------------------------------------ crossover
def single_point_crossover(a: torch.Tensor, b: torch.Tensor, points: torch.Tensor | None = None, generator=None):
    """Per pair a cut point in [1, D - 1]: child1 = a[:p] + b[p:], child2 = b[:p] + a[p:]."""
    d = a.shape[-1]
    if d <= 1:
        return a.clone(), b.clone()
    if points is None:
        points = torch.randint(1, d, a.shape[:-1], generator=generator).to(a.device)
    m = torch.arange(d, device=a.device) < points[..., None]
    return torch.where(m, a, b), torch.where(m, b, a)


def uniform_crossover(a, b, u: torch.Tensor | None = None, generator=None):
    """Per gene a draw u: u < 0.5 keeps (a, b), else swaps."""
    if u is None:
        u = torch.rand(a.shape, generator=generator, dtype=torch.float64).to(a.device)
    m = u < 0.5
    return torch.where(m, a, b), torch.where(m, b, a)


def blx_alpha_crossover(a, b, alpha: float, u1: torch.Tensor | None = None, u2: torch.Tensor | None = None,
                        generator=None):
    """Both children uniform in [min - alpha range, max + alpha range] per gene."""
    lo, hi = torch.minimum(a, b), torch.maximum(a, b)
    r = hi - lo
    lo, hi = lo - alpha * r, hi + alpha * r
    if u1 is None:
        u1 = torch.rand(a.shape, generator=generator, dtype=torch.float64).to(a.device)
    if u2 is None:
        u2 = torch.rand(a.shape, generator=generator, dtype=torch.float64).to(a.device)
    return lo + u1 * (hi - lo), lo + u2 * (hi - lo)


def sbx_crossover(a, b, eta_c: float, u: torch.Tensor | None = None, generator=None):
    """Simulated binary crossover (Deb and Agrawal 1995): spread beta = (2u)^(1/(eta+1)) for u <= 0.5,
    else (1 / (2 (1 - u)))^(1/(eta+1)); children 0.5 ((1 +- beta) a + (1 -+ beta) b)."""
    if u is None:
        u = torch.rand(a.shape, generator=generator, dtype=torch.float64).to(a.device)
    e = 1.0 / (eta_c + 1.0)
    beta = torch.where(u <= 0.5, (2.0 * u) ** e, (1.0 / (2.0 * (1.0 - u))) ** e)
    return 0.5 * ((1 + beta) * a + (1 - beta) * b), 0.5 * ((1 - beta) * a + (1 + beta) * b)


# ------------------------------------------------------------------------------------------ ranking / stats
def rank_fitness(fitnesses) -> list[int]:
    """Indices from best (highest) to worst; ties keep index order."""
    f = torch.as_tensor(fitnesses, dtype=torch.float64)
    return torch.sort(f, descending=True, stable=True).indices.tolist()


@dataclass
class FitnessStats:
    best: float = 0.0
    mean: float = 0.0
    median: float = 0.0
    worst: float = 0.0

    @classmethod
    def from_fitnesses(cls, fits) -> "FitnessStats":
        f = torch.as_tensor(fits, dtype=torch.float64).reshape(-1)
        if f.numel() == 0:
            return cls()
        s = torch.sort(f).values
        n = s.numel()
        med = float(s[n // 2]) if n % 2 else float((s[n // 2 - 1] + s[n // 2]) * 0.5)
        return cls(float(s[-1]), float(s.mean()), med, float(s[0]))


@dataclass
class TerminationConfig:
    max_generations: int = 100
    patience: int | None = 20
    min_fitness_delta: float = 1e-4
    target_fitness: float | None = None


@dataclass
class TerminationTracker:
    best_fitness: float = -math.inf
    generations_without_improvement: int = 0

    def update(self, current_best: float, config: TerminationConfig) -> bool:
        """Improvement means beating the best by more than min_fitness_delta; stop on reaching the
        target or after ``patience`` generations without improvement."""
        if current_best > self.best_fitness + config.min_fitness_delta:
            self.best_fitness, self.generations_without_improvement = current_best, 0
        else:
            self.generations_without_improvement += 1
        if config.target_fitness is not None and current_best >= config.target_fitness:
            return True
        return config.patience is not None and self.generations_without_improvement >= config.patience


def evaluate_population_parallel(population: torch.Tensor, fitness_fn, chunk: int = 0) -> torch.Tensor:
    """Fitness of every genome: one batched call of ``fitness_fn`` on [P, D] (or chunks of it)."""
    if not chunk or population.shape[0] <= chunk:
        return fitness_fn(population)
    return torch.cat([fitness_fn(population[i:i + chunk]) for i in range(0, population.shape[0], chunk)])


# ------------------------------------------------------------------------------------------ HyperNEAT
_ACT = {
    "linear": lambda x: x,
    "sigmoid": torch.sigmoid,
    "gaussian": lambda x: torch.exp(-x * x),
    "sine": torch.sin,
    "abs": torch.abs,
}


@dataclass
class CppnNode:
    activation: str = "linear"
    bias: float = 0.0
    inputs: list = field(default_factory=list)  # (source index, weight); sources < 5 are the coordinate inputs


class Cppn:
    """Compositional pattern-producing network over the inputs (x1, y1, x2, y2, d) with d the distance
    between the two points; nodes are evaluated in order (each reads inputs and earlier nodes), the
    last node is the output. An empty network is gaussian(d) - 0.5."""

    N_IN = 5

    def __init__(self, nodes: list[CppnNode] | None = None):
        self.nodes = list(nodes or [])

    @classmethod
    def default(cls) -> "Cppn":
        return cls([CppnNode("gaussian", 0.0, [(4, 1.0)]), CppnNode("linear", -0.5, [(5, 1.0)])])

    def query(self, x1, y1, x2, y2) -> torch.Tensor:
        x1, y1, x2, y2 = (torch.as_tensor(v, dtype=torch.float64) for v in (x1, y1, x2, y2))
        d = torch.sqrt((x2 - x1) ** 2 + (y2 - y1) ** 2)
        if not self.nodes:
            return torch.exp(-d * d) - 0.5
        vals = list(torch.broadcast_tensors(x1, y1, x2, y2, d))
        for n in self.nodes:
            s = torch.full_like(vals[0], n.bias)
            for src, w in n.inputs:
                s = s + w * vals[src]
            vals.append(_ACT[n.activation](s))
        return vals[-1]

    def mutate(self, generator=None, sigma: float = 0.1) -> "Cppn":
        """A copy with Gaussian noise on every bias and connection weight."""
        def nz():
            return float(torch.randn((), generator=generator)) * sigma
        return Cppn([CppnNode(n.activation, n.bias + nz(), [(s, w + nz()) for s, w in n.inputs]) for n in self.nodes])


def _grid(w: int, h: int) -> torch.Tensor:
    xs = torch.linspace(-1.0, 1.0, w, dtype=torch.float64) if w > 1 else torch.zeros(1, dtype=torch.float64)
    ys = torch.linspace(-1.0, 1.0, h, dtype=torch.float64) if h > 1 else torch.zeros(1, dtype=torch.float64)
    yy, xx = torch.meshgrid(ys, xs, indexing="ij")
    return torch.stack([xx.reshape(-1), yy.reshape(-1)], 1)  # row-major: y outer, x inner


@dataclass
class SubstrateConfig:
    input_width: int = 3
    input_height: int = 3
    output_width: int = 3
    output_height: int = 3


class SubstrateGrid2D:
    """Input and output neurons on [-1, 1]^2 grids (a single row or column sits at 0)."""

    def __init__(self, in_w: int, in_h: int, out_w: int, out_h: int):
        self.in_coords, self.out_coords = _grid(in_w, in_h), _grid(out_w, out_h)

    def generate_weight_matrix(self, cppn: Cppn, threshold: float = 0.0) -> torch.Tensor:
        """W[out, in] = cppn(x_in, y_in, x_out, y_out) for all pairs at once; |w| <= threshold -> 0."""
        o, i = self.out_coords, self.in_coords
        w = cppn.query(i[None, :, 0], i[None, :, 1], o[:, None, 0], o[:, None, 1])
        return torch.where(w.abs() > threshold, w, torch.zeros_like(w)) if threshold > 0 else w


@dataclass
class EvoCheckpoint:
    generation: int
    population: torch.Tensor
    fitnesses: torch.Tensor
    best_genome: torch.Tensor
    best_fitness: float

    def save(self, path: str) -> None:
        torch.save(self.__dict__, path)

    @classmethod
    def load(cls, path: str) -> "EvoCheckpoint":
        return cls(**torch.load(path, weights_only=True))
