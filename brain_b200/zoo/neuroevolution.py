"""Neuroevolution: real-valued genomes, selection (tournament, roulette, rank), crossover (uniform,
one-point, blend), Gaussian mutation, a generational genetic algorithm with elitism, the (1+1)-ES with the
1/5th success rule, CMA-ES, and evolving the flat weight vector of a network.

Reference: crates/brain-neuroevolution. GA (ga/mod.rs:21-120, termination ga/termination.rs),
selection (selection.rs:11-100), crossover (crossover.rs), mutation (mutation.rs), (1+1)-ES
(es/es1p1.rs), CMA-ES (es/cmaes.rs:12-200), weight evolution (neuro/weights.rs).

Whole populations are evaluated as one batch where the fitness function accepts a [P, D] tensor
(``batched=True``), so a network population can be scored with one batched forward on the GPU. CMA-ES
follows Hansen's tutorial (2016) update equations.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


def _fitness(fn, pop: torch.Tensor, batched: bool) -> torch.Tensor:
    if batched:
        return torch.as_tensor(fn(pop), dtype=torch.float64).reshape(-1)
    return torch.tensor([float(fn(g)) for g in pop], dtype=torch.float64)


def tournament_select(pop, fit, k: int, n: int, generator=None):
    idx = torch.randint(0, pop.shape[0], (n, k), generator=generator)
    win = idx.gather(1, fit[idx].argmax(1, keepdim=True)).squeeze(1)
    return pop[win]


def roulette_wheel_select(pop, fit, n: int, generator=None):
    w = fit - fit.min() + 1e-12
    return pop[torch.multinomial(w / w.sum(), n, replacement=True, generator=generator)]


def rank_based_select(pop, fit, n: int, generator=None):
    ranks = torch.empty_like(fit)
    ranks[fit.argsort()] = torch.arange(1, fit.numel() + 1, dtype=fit.dtype)
    return pop[torch.multinomial(ranks / ranks.sum(), n, replacement=True, generator=generator)]


def uniform_crossover(a, b, generator=None):
    m = torch.rand(a.shape, generator=generator) < 0.5
    return torch.where(m, a, b)


def one_point_crossover(a, b, generator=None):
    cut = torch.randint(1, a.shape[-1], (a.shape[0], 1), generator=generator)
    pos = torch.arange(a.shape[-1])[None]
    return torch.where(pos < cut, a, b)


def blend_crossover(a, b, alpha: float = 0.5, generator=None):
    """BLX-α: uniform in [min − αd, max + αd] per gene."""
    lo, hi = torch.minimum(a, b), torch.maximum(a, b)
    d = hi - lo
    return lo - alpha * d + torch.rand(a.shape, generator=generator, dtype=a.dtype) * (1 + 2 * alpha) * d


def gaussian_mutation(pop, rate: float, sigma: float, generator=None):
    m = torch.rand(pop.shape, generator=generator) < rate
    return pop + m * torch.randn(pop.shape, generator=generator, dtype=pop.dtype) * sigma


@dataclass
class GaConfig:
    population: int = 64
    genome_len: int = 8
    generations: int = 100
    elite: int = 2
    tournament: int = 3
    mutation_rate: float = 0.1
    mutation_sigma: float = 0.3
    crossover: str = "uniform"
    selection: str = "tournament"
    init_scale: float = 1.0
    target_fitness: float | None = None
    patience: int = 0


@dataclass
class GaResult:
    best: torch.Tensor
    best_fitness: float
    history: list
    generations: int


class Ga:
    """Maximises ``fitness_fn``."""

    def __init__(self, config: GaConfig, seed: int = 0):
        self.c = config
        self.gen = torch.Generator().manual_seed(seed)

    def run(self, fitness_fn, batched: bool = False) -> GaResult:
        c, g = self.c, self.gen
        pop = torch.randn(c.population, c.genome_len, generator=g, dtype=torch.float64) * c.init_scale
        hist, best, best_f, stale = [], None, -math.inf, 0
        for gen in range(c.generations):
            fit = _fitness(fitness_fn, pop, batched)
            i = int(fit.argmax())
            if fit[i] > best_f + 1e-12:
                best, best_f, stale = pop[i].clone(), float(fit[i]), 0
            else:
                stale += 1
            hist.append(float(fit.max()))
            if (c.target_fitness is not None and best_f >= c.target_fitness) or (c.patience and stale >= c.patience):
                return GaResult(best, best_f, hist, gen + 1)
            elite = pop[fit.argsort(descending=True)[:c.elite]]
            n = c.population - c.elite
            if c.selection == "roulette":
                pa, pb = roulette_wheel_select(pop, fit, n, g), roulette_wheel_select(pop, fit, n, g)
            elif c.selection == "rank":
                pa, pb = rank_based_select(pop, fit, n, g), rank_based_select(pop, fit, n, g)
            else:
                pa, pb = tournament_select(pop, fit, c.tournament, n, g), tournament_select(pop, fit, c.tournament, n, g)
            cross = {"uniform": uniform_crossover, "one_point": one_point_crossover, "blend": blend_crossover}[c.crossover]
            kids = gaussian_mutation(cross(pa, pb, generator=g), c.mutation_rate, c.mutation_sigma, g)
            pop = torch.cat([elite, kids])
        fit = _fitness(fitness_fn, pop, batched)
        i = int(fit.argmax())
        if fit[i] > best_f:
            best, best_f = pop[i].clone(), float(fit[i])
        return GaResult(best, best_f, hist, c.generations)


def es_one_plus_one(fitness_fn, x0: torch.Tensor, sigma: float = 0.5, iters: int = 500, seed: int = 0):
    """(1+1)-ES maximising ``fitness_fn`` with the 1/5th success rule (σ ×1.5 / ×0.82 per 10-step window)."""
    g = torch.Generator().manual_seed(seed)
    x, fx = x0.double().clone(), float(fitness_fn(x0.double()))
    succ = 0
    for it in range(1, iters + 1):
        y = x + sigma * torch.randn(x.shape, generator=g, dtype=torch.float64)
        fy = float(fitness_fn(y))
        if fy >= fx:
            x, fx = y, fy
            succ += 1
        if it % 10 == 0:
            sigma *= 1.5 if succ > 2 else 0.82
            succ = 0
    return x, fx


@dataclass
class CmaesConfig:
    dim: int
    sigma: float = 0.5
    population: int = 0
    max_iters: int = 200
    tol: float = 1e-10


class Cmaes:
    """Maximises ``fitness_fn`` (internally minimises its negation) with rank-μ and rank-one covariance
    updates, cumulative step-size adaptation and evolution paths."""

    def __init__(self, config: CmaesConfig, seed: int = 0, x0: torch.Tensor | None = None):
        self.c = config
        self.gen = torch.Generator().manual_seed(seed)
        self.mean = torch.zeros(config.dim, dtype=torch.float64) if x0 is None else x0.double().clone()

    def optimize(self, fitness_fn, batched: bool = False):
        n = self.c.dim
        lam = self.c.population or 4 + int(3 * math.log(n))
        mu = lam // 2
        w = math.log(mu + 0.5) - torch.log(torch.arange(1, mu + 1, dtype=torch.float64))
        w = w / w.sum()
        mueff = float(1 / (w ** 2).sum())
        cc = (4 + mueff / n) / (n + 4 + 2 * mueff / n)
        cs = (mueff + 2) / (n + mueff + 5)
        c1 = 2 / ((n + 1.3) ** 2 + mueff)
        cmu = min(1 - c1, 2 * (mueff - 2 + 1 / mueff) / ((n + 2) ** 2 + mueff))
        damps = 1 + 2 * max(0.0, math.sqrt((mueff - 1) / (n + 1)) - 1) + cs
        chin = math.sqrt(n) * (1 - 1 / (4 * n) + 1 / (21 * n * n))
        C = torch.eye(n, dtype=torch.float64)
        pc, ps = torch.zeros(n, dtype=torch.float64), torch.zeros(n, dtype=torch.float64)
        sigma, m = self.c.sigma, self.mean
        best, best_f = m.clone(), -math.inf
        for it in range(self.c.max_iters):
            evals, B = torch.linalg.eigh(C)
            D = evals.clamp(min=1e-20).sqrt()
            z = torch.randn(lam, n, generator=self.gen, dtype=torch.float64)
            y = z @ (B * D).t()
            x = m + sigma * y
            f = _fitness(fitness_fn, x, batched)
            order = f.argsort(descending=True)
            if f[order[0]] > best_f:
                best, best_f = x[order[0]].clone(), float(f[order[0]])
            ysel = y[order[:mu]]
            yw = (w[:, None] * ysel).sum(0)
            m = m + sigma * yw
            Cinvsqrt = (B / D) @ B.t()
            ps = (1 - cs) * ps + math.sqrt(cs * (2 - cs) * mueff) * (Cinvsqrt @ yw)
            hsig = float(ps.norm() / math.sqrt(1 - (1 - cs) ** (2 * (it + 1))) / chin < 1.4 + 2 / (n + 1))
            pc = (1 - cc) * pc + hsig * math.sqrt(cc * (2 - cc) * mueff) * yw
            rank_mu = (w[:, None, None] * ysel[:, :, None] * ysel[:, None, :]).sum(0)
            C = ((1 - c1 - cmu) * C + c1 * (torch.outer(pc, pc) + (1 - hsig) * cc * (2 - cc) * C) + cmu * rank_mu)
            C = 0.5 * (C + C.t())
            sigma *= math.exp((cs / damps) * (float(ps.norm()) / chin - 1))
            if sigma * float(D.max()) < self.c.tol:
                break
        self.mean = m
        return best, best_f


def get_flat_weights(model: torch.nn.Module) -> torch.Tensor:
    return torch.cat([p.detach().reshape(-1).double().cpu() for p in model.parameters()])


def set_flat_weights(model: torch.nn.Module, flat: torch.Tensor) -> None:
    off = 0
    with torch.no_grad():
        for p in model.parameters():
            p.copy_(flat[off:off + p.numel()].view_as(p).to(p.dtype))
            off += p.numel()


def evolve_network(model: torch.nn.Module, fitness_of_model, config: GaConfig | None = None, seed: int = 0):
    """GA over the model's flat weights; leaves the best weights loaded and returns the GaResult."""
    n = get_flat_weights(model).numel()
    cfg = config or GaConfig()
    cfg.genome_len = n

    def fit(genome):
        set_flat_weights(model, genome)
        return fitness_of_model(model)

    res = Ga(cfg, seed).run(fit)
    set_flat_weights(model, res.best)
    return res
