"""Optimizer family with the reference's names and update rules (crates/brain-optim/src/).

``Optimizer`` keeps the reference trait's surface: ``step() -> StepInfo{grad_norm, param_norm, lr}``
(optimizer/mod.rs:70-130), ``zero_grad``, ``get_lr``/``set_lr``, parameter groups and
``state_dict``/``load_state_dict``. Adam/AdamW/SGD run the fused CUDA kernels (``csrc/optim.cu``)
on each float32 CUDA parameter; everything else is written with tensor ops.

AdamW order follows crates/brain-optim/src/adam/mod.rs:128-200: effective decay ``max(group.wd,
cfg.wd)``, decoupled decay applied to p before the moment update, bias correction by powers of
beta, optional AMSGrad. A non-finite gradient makes ``step`` raise (the reference returns an
error) unless ``skip_nonfinite`` is set, in which case the step is skipped.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops import optim_kernels as K


@dataclass
class StepInfo:
    grad_norm: float
    param_norm: float
    lr: float


class NonFiniteGradient(FloatingPointError):
    pass


class Optimizer:
    defaults: dict = {}

    def __init__(self, params, **defaults):
        params = list(params)
        if params and isinstance(params[0], dict):
            groups = params
        else:
            groups = [{"params": params}]
        self.param_groups = []
        for g in groups:
            d = dict(self.defaults)
            d.update(defaults)
            d.update({k: v for k, v in g.items() if k != "params"})
            d["params"] = [p for p in g["params"]]
            self.param_groups.append(d)
        self.state: dict = {}
        self.step_count = 0
        self.skip_nonfinite = False
        self.compute_norms = True

    # reference-style API
    def get_lr(self) -> float:
        return self.param_groups[0]["lr"]

    def set_lr(self, lr: float) -> None:
        for g in self.param_groups:
            g["lr"] = lr

    def zero_grad(self, set_to_none: bool = True) -> None:
        for g in self.param_groups:
            for p in g["params"]:
                if set_to_none:
                    p.grad = None
                elif p.grad is not None:
                    p.grad.zero_()

    def _params(self):
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is not None:
                    yield g, p

    @torch.no_grad()
    def step(self, closure=None) -> StepInfo:
        loss = closure() if closure is not None else None  # noqa: F841
        gn2 = 0.0
        finite = True
        if self.compute_norms or not self.skip_nonfinite:
            for _, p in self._params():
                g = p.grad.float()
                if not torch.isfinite(g).all():
                    finite = False
                gn2 += float(g.pow(2).sum())
        if not finite:
            if self.skip_nonfinite:
                return StepInfo(float("nan"), self._param_norm(), self.get_lr())
            raise NonFiniteGradient("non-finite gradient")
        self.step_count += 1
        for g, p in self._params():
            self._update(p, p.grad, g, self.state.setdefault(id(p), {}))
        return StepInfo(math.sqrt(gn2), self._param_norm(), self.get_lr())

    def _param_norm(self) -> float:
        if not self.compute_norms:
            return 0.0
        return math.sqrt(sum(float(p.detach().float().pow(2).sum()) for g in self.param_groups for p in g["params"]))

    def _update(self, p, grad, group, state):  # pragma: no cover - abstract
        raise NotImplementedError

    def state_dict(self) -> dict:
        idx = {}
        for g in self.param_groups:
            for p in g["params"]:
                idx[id(p)] = len(idx)
        st = {idx[k]: {n: (v.clone() if isinstance(v, torch.Tensor) else v) for n, v in s.items()}
              for k, s in self.state.items() if k in idx}
        groups = [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups]
        return {"state": st, "param_groups": groups, "step": self.step_count}

    def load_state_dict(self, sd: dict) -> None:
        plist = [p for g in self.param_groups for p in g["params"]]
        self.state = {id(plist[int(i)]): {n: (v.clone() if isinstance(v, torch.Tensor) else v) for n, v in s.items()}
                      for i, s in sd["state"].items()}
        for g, sg in zip(self.param_groups, sd["param_groups"]):
            g.update(sg)
        self.step_count = sd.get("step", 0)


def _fused_ok(p, grad) -> bool:
    return p.is_cuda and p.dtype == torch.float32 and p.is_contiguous() and grad.is_contiguous()


class Adam(Optimizer):
    defaults = {"lr": 1e-3, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 0.0, "amsgrad": False,
                "decoupled": False}

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, amsgrad=False, **kw):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=amsgrad, **kw)

    def _update(self, p, grad, group, state):
        if not state:
            state["step"] = 0
            state["exp_avg"] = torch.zeros_like(p, dtype=torch.float32)
            state["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32)
            if group["amsgrad"]:
                state["max_exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32)
        state["step"] += 1
        b1, b2 = group["betas"]
        lr, eps, wd = group["lr"], group["eps"], group["weight_decay"]
        if not group["decoupled"] and wd:
            grad = grad + wd * p  # classic L2 (Adam) folds decay into the gradient
            wd = 0.0
        if _fused_ok(p, grad):
            K.adamw_(p.view(-1), state["exp_avg"].view(-1), state["exp_avg_sq"].view(-1), grad.reshape(-1), lr=lr,
                     beta1=b1, beta2=b2, eps=eps, weight_decay=wd, step=state["step"],
                     vmax=state.get("max_exp_avg_sq", None) if group["amsgrad"] else None)
            return
        pf = p.data.float()
        K.adamw_(pf, state["exp_avg"], state["exp_avg_sq"], grad.float(), lr=lr, beta1=b1, beta2=b2, eps=eps,
                 weight_decay=wd, step=state["step"], vmax=state.get("max_exp_avg_sq"))
        p.data.copy_(pf)


class AdamW(Adam):
    defaults = dict(Adam.defaults, weight_decay=0.01, decoupled=True)

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, amsgrad=False, **kw):
        Optimizer.__init__(self, params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=amsgrad,
                           decoupled=True, **kw)


class SGD(Optimizer):
    defaults = {"lr": 0.01, "momentum": 0.0, "dampening": 0.0, "weight_decay": 0.0, "nesterov": False}

    def __init__(self, params, lr=0.01, momentum=0.0, dampening=0.0, weight_decay=0.0, nesterov=False):
        super().__init__(params, lr=lr, momentum=momentum, dampening=dampening, weight_decay=weight_decay,
                         nesterov=nesterov)

    def _update(self, p, grad, group, state):
        first = "momentum_buffer" not in state
        if group["momentum"] and first:
            state["momentum_buffer"] = torch.zeros_like(p, dtype=torch.float32)
        buf = state.get("momentum_buffer")
        kw = dict(lr=group["lr"], momentum=group["momentum"], dampening=group["dampening"],
                  weight_decay=group["weight_decay"], nesterov=group["nesterov"], first=first)
        if _fused_ok(p, grad):
            K.sgd_(p.view(-1), None if buf is None else buf.view(-1), grad.reshape(-1), **kw)
        else:
            pf = p.data.float()
            K.sgd_(pf, buf, grad.float(), **kw)
            p.data.copy_(pf)


class Adamax(Optimizer):
    defaults = {"lr": 2e-3, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        if not st:
            st.update(step=0, m=torch.zeros_like(p), u=torch.zeros_like(p))
        st["step"] += 1
        b1, b2 = group["betas"]
        if group["weight_decay"]:
            g = g + group["weight_decay"] * p
        st["m"].mul_(b1).add_(g, alpha=1 - b1)
        st["u"] = torch.maximum(st["u"] * b2, g.abs() + group["eps"])
        p.sub_(group["lr"] / (1 - b1 ** st["step"]) * st["m"] / st["u"])


class NAdam(Optimizer):
    defaults = {"lr": 2e-3, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        if not st:
            st.update(step=0, m=torch.zeros_like(p), v=torch.zeros_like(p))
        st["step"] += 1
        t = st["step"]
        b1, b2 = group["betas"]
        if group["weight_decay"]:
            g = g + group["weight_decay"] * p
        st["m"].mul_(b1).add_(g, alpha=1 - b1)
        st["v"].mul_(b2).addcmul_(g, g, value=1 - b2)
        mh = (b1 * st["m"] / (1 - b1 ** (t + 1))) + ((1 - b1) * g / (1 - b1 ** t))
        vh = st["v"] / (1 - b2 ** t)
        p.sub_(group["lr"] * mh / (vh.sqrt() + group["eps"]))


Nadam = NAdam


class RAdam(Optimizer):
    defaults = {"lr": 1e-3, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        if not st:
            st.update(step=0, m=torch.zeros_like(p), v=torch.zeros_like(p))
        st["step"] += 1
        t = st["step"]
        b1, b2 = group["betas"]
        if group["weight_decay"]:
            g = g + group["weight_decay"] * p
        st["m"].mul_(b1).add_(g, alpha=1 - b1)
        st["v"].mul_(b2).addcmul_(g, g, value=1 - b2)
        mh = st["m"] / (1 - b1 ** t)
        rho_inf = 2 / (1 - b2) - 1
        rho = rho_inf - 2 * t * b2 ** t / (1 - b2 ** t)
        if rho > 5:
            r = math.sqrt((rho - 4) * (rho - 2) * rho_inf / ((rho_inf - 4) * (rho_inf - 2) * rho))
            vh = (st["v"] / (1 - b2 ** t)).sqrt()
            p.sub_(group["lr"] * r * mh / (vh + group["eps"]))
        else:
            p.sub_(group["lr"] * mh)


class Lamb(Optimizer):
    defaults = {"lr": 1e-3, "betas": (0.9, 0.999), "eps": 1e-6, "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        if not st:
            st.update(step=0, m=torch.zeros_like(p), v=torch.zeros_like(p))
        st["step"] += 1
        t = st["step"]
        b1, b2 = group["betas"]
        st["m"].mul_(b1).add_(g, alpha=1 - b1)
        st["v"].mul_(b2).addcmul_(g, g, value=1 - b2)
        upd = (st["m"] / (1 - b1 ** t)) / ((st["v"] / (1 - b2 ** t)).sqrt() + group["eps"])
        upd = upd + group["weight_decay"] * p
        wn, un = p.norm(), upd.norm()
        trust = (wn / un) if (wn > 0 and un > 0) else torch.tensor(1.0, device=p.device)
        p.sub_(group["lr"] * trust * upd)


class Lion(Optimizer):
    defaults = {"lr": 1e-4, "betas": (0.9, 0.99), "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        if not st:
            st["m"] = torch.zeros_like(p)
        b1, b2 = group["betas"]
        p.mul_(1 - group["lr"] * group["weight_decay"])
        upd = (st["m"] * b1 + g * (1 - b1)).sign()
        p.sub_(group["lr"] * upd)
        st["m"].mul_(b2).add_(g, alpha=1 - b2)


class NovoGrad(Optimizer):
    defaults = {"lr": 1e-3, "betas": (0.95, 0.98), "eps": 1e-8, "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        b1, b2 = group["betas"]
        n = g.pow(2).sum()
        if not st:
            st.update(v=n.clone(), m=torch.zeros_like(p))
        else:
            st["v"] = b2 * st["v"] + (1 - b2) * n
        gg = g / (st["v"].sqrt() + group["eps"]) + group["weight_decay"] * p
        st["m"].mul_(b1).add_(gg)
        p.sub_(group["lr"] * st["m"])


class RMSprop(Optimizer):
    defaults = {"lr": 1e-2, "alpha": 0.99, "eps": 1e-8, "weight_decay": 0.0, "momentum": 0.0, "centered": False}

    def _update(self, p, g, group, st):
        if not st:
            st.update(sq=torch.zeros_like(p), buf=torch.zeros_like(p), gavg=torch.zeros_like(p))
        if group["weight_decay"]:
            g = g + group["weight_decay"] * p
        a = group["alpha"]
        st["sq"].mul_(a).addcmul_(g, g, value=1 - a)
        avg = st["sq"]
        if group["centered"]:
            st["gavg"].mul_(a).add_(g, alpha=1 - a)
            avg = avg - st["gavg"].pow(2)
        denom = avg.sqrt() + group["eps"]
        if group["momentum"]:
            st["buf"].mul_(group["momentum"]).addcdiv_(g, denom)
            p.sub_(group["lr"] * st["buf"])
        else:
            p.addcdiv_(g, denom, value=-group["lr"])


class Adagrad(Optimizer):
    defaults = {"lr": 1e-2, "eps": 1e-10, "weight_decay": 0.0, "initial_accumulator_value": 0.0}

    def _update(self, p, g, group, st):
        if not st:
            st["sum"] = torch.full_like(p, group["initial_accumulator_value"])
        if group["weight_decay"]:
            g = g + group["weight_decay"] * p
        st["sum"].addcmul_(g, g)
        p.addcdiv_(g, st["sum"].sqrt() + group["eps"], value=-group["lr"])


class Adadelta(Optimizer):
    defaults = {"lr": 1.0, "rho": 0.9, "eps": 1e-6, "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        if not st:
            st.update(sq=torch.zeros_like(p), acc=torch.zeros_like(p))
        if group["weight_decay"]:
            g = g + group["weight_decay"] * p
        rho, eps = group["rho"], group["eps"]
        st["sq"].mul_(rho).addcmul_(g, g, value=1 - rho)
        d = (st["acc"] + eps).sqrt() / (st["sq"] + eps).sqrt() * g
        st["acc"].mul_(rho).addcmul_(d, d, value=1 - rho)
        p.sub_(group["lr"] * d)


class Adafactor(Optimizer):
    """Factored second moment for matrices (row/column statistics), full for vectors."""
    defaults = {"lr": 1e-3, "beta2_decay": -0.8, "eps": 1e-30, "clip_threshold": 1.0, "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        if not st:
            st["step"] = 0
            if p.dim() >= 2:
                st["r"] = torch.zeros(p.shape[:-1], device=p.device)
                st["c"] = torch.zeros(p.shape[:-2] + p.shape[-1:], device=p.device)
            else:
                st["v"] = torch.zeros_like(p)
        st["step"] += 1
        b2 = 1.0 - st["step"] ** group["beta2_decay"]
        g2 = g.float().pow(2) + group["eps"]
        if p.dim() >= 2:
            st["r"].mul_(b2).add_(g2.mean(-1), alpha=1 - b2)
            st["c"].mul_(b2).add_(g2.mean(-2), alpha=1 - b2)
            v = st["r"].unsqueeze(-1) * st["c"].unsqueeze(-2) / st["r"].mean(-1, keepdim=True).unsqueeze(-1)
        else:
            st["v"].mul_(b2).add_(g2, alpha=1 - b2)
            v = st["v"]
        u = g / v.sqrt()
        u = u / max(1.0, float(u.pow(2).mean().sqrt()) / group["clip_threshold"])
        if group["weight_decay"]:
            p.mul_(1 - group["lr"] * group["weight_decay"])
        p.sub_(group["lr"] * u)


class Adan(Optimizer):
    defaults = {"lr": 1e-3, "betas": (0.98, 0.92, 0.99), "eps": 1e-8, "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        b1, b2, b3 = group["betas"]
        if not st:
            st.update(m=torch.zeros_like(p), v=torch.zeros_like(p), n=torch.zeros_like(p), prev=g.clone())
        diff = g - st["prev"]
        st["m"].mul_(b1).add_(g, alpha=1 - b1)
        st["v"].mul_(b2).add_(diff, alpha=1 - b2)
        z = g + b2 * diff
        st["n"].mul_(b3).addcmul_(z, z, value=1 - b3)
        upd = (st["m"] + b2 * st["v"]) / (st["n"].sqrt() + group["eps"])
        p.sub_(group["lr"] * upd).div_(1 + group["lr"] * group["weight_decay"])
        st["prev"] = g.clone()


class Sophia(Optimizer):
    """Sophia-G style: EMA of gradients over a clipped diagonal curvature estimate (|g|^2 EMA)."""
    defaults = {"lr": 1e-4, "betas": (0.965, 0.99), "rho": 0.04, "eps": 1e-12, "weight_decay": 0.0}

    def _update(self, p, g, group, st):
        b1, b2 = group["betas"]
        if not st:
            st.update(m=torch.zeros_like(p), h=torch.zeros_like(p))
        st["m"].mul_(b1).add_(g, alpha=1 - b1)
        st["h"].mul_(b2).addcmul_(g, g, value=1 - b2)
        p.mul_(1 - group["lr"] * group["weight_decay"])
        ratio = (st["m"].abs() / (group["rho"] * st["h"] + group["eps"])).clamp(max=1.0)
        p.sub_(group["lr"] * st["m"].sign() * ratio)


class Muon(Optimizer):
    """Momentum orthogonalised by Newton-Schulz iterations for matrices (Adam-free for 2-D params)."""
    defaults = {"lr": 0.02, "momentum": 0.95, "nesterov": True, "ns_steps": 5, "weight_decay": 0.0}

    @staticmethod
    def _ns(gm, steps):
        a, b, c = 3.4445, -4.7750, 2.0315
        x = gm / (gm.norm() + 1e-7)
        tr = x.shape[0] > x.shape[1]
        if tr:
            x = x.t()
        for _ in range(steps):
            A = x @ x.t()
            x = a * x + (b * A + c * A @ A) @ x
        return x.t() if tr else x

    def _update(self, p, g, group, st):
        if "buf" not in st:
            st["buf"] = torch.zeros_like(p)
        st["buf"].mul_(group["momentum"]).add_(g)
        u = g + group["momentum"] * st["buf"] if group["nesterov"] else st["buf"]
        if p.dim() >= 2:
            u = self._ns(u.reshape(p.shape[0], -1).float(), group["ns_steps"]).reshape(p.shape)
            u = u * max(1.0, p.shape[0] / p[0].numel()) ** 0.5
        p.mul_(1 - group["lr"] * group["weight_decay"])
        p.sub_(group["lr"] * u.to(p.dtype))


class SAM:
    """Sharpness-aware minimisation wrapper: ascend to w + rho g/|g|, recompute grads, descend."""

    def __init__(self, base: Optimizer, rho: float = 0.05):
        self.base, self.rho = base, rho
        self._e = {}

    @torch.no_grad()
    def first_step(self):
        norm = math.sqrt(sum(float(p.grad.pow(2).sum()) for _, p in self.base._params()))
        for _, p in self.base._params():
            e = p.grad * (self.rho / (norm + 1e-12))
            p.add_(e)
            self._e[id(p)] = e

    @torch.no_grad()
    def second_step(self):
        for _, p in self.base._params():
            p.sub_(self._e.pop(id(p), 0))
        return self.base.step()

    def zero_grad(self):
        self.base.zero_grad()


class Lookahead:
    def __init__(self, base: Optimizer, k: int = 5, alpha: float = 0.5):
        self.base, self.k, self.alpha = base, k, alpha
        self.slow = {id(p): p.detach().clone() for g in base.param_groups for p in g["params"]}
        self.n = 0

    @torch.no_grad()
    def step(self):
        info = self.base.step()
        self.n += 1
        if self.n % self.k == 0:
            for g in self.base.param_groups:
                for p in g["params"]:
                    s = self.slow[id(p)]
                    s.add_(p - s, alpha=self.alpha)
                    p.copy_(s)
        return info

    def zero_grad(self):
        self.base.zero_grad()


class EMA:
    """Exponential moving average of parameters (shadow weights)."""

    def __init__(self, params, decay: float = 0.999):
        self.decay = decay
        self.params = list(params)
        self.shadow = [p.detach().clone().float() for p in self.params]

    @torch.no_grad()
    def update(self):
        for s, p in zip(self.shadow, self.params):
            s.mul_(self.decay).add_(p.detach().float(), alpha=1 - self.decay)

    @torch.no_grad()
    def copy_to(self, params=None):
        for s, p in zip(self.shadow, params or self.params):
            p.copy_(s.to(p.dtype))


class SWA(EMA):
    """Stochastic weight averaging (uniform average of snapshots)."""

    def __init__(self, params):
        super().__init__(params, 0.0)
        self.n = 0

    @torch.no_grad()
    def update(self):
        self.n += 1
        for s, p in zip(self.shadow, self.params):
            s.add_((p.detach().float() - s) / self.n)


# ------------------------------------------------------------------ clipping
@torch.no_grad()
def clip_grad_norm_(params, max_norm: float, norm_type: float = 2.0) -> float:
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return 0.0
    if norm_type == float("inf"):
        total = max(float(g.abs().max()) for g in grads)
    else:
        total = sum(float(g.float().norm(norm_type)) ** norm_type for g in grads) ** (1.0 / norm_type)
    coef = max_norm / (total + 1e-6)
    if coef < 1.0:
        for g in grads:
            g.mul_(coef)
    return total


@torch.no_grad()
def clip_grad_value_(params, clip: float) -> None:
    for p in params:
        if p.grad is not None:
            p.grad.clamp_(-clip, clip)


@torch.no_grad()
def adaptive_clip_grad_(params, clip: float = 0.01, eps: float = 1e-3) -> None:
    """AGC: clip each gradient to clip * max(|w|, eps) (unit-wise over rows)."""
    for p in params:
        if p.grad is None:
            continue
        dims = tuple(range(1, p.dim())) if p.dim() > 1 else (0,)
        wn = p.detach().float().norm(dim=dims, keepdim=True).clamp_min(eps)
        gn = p.grad.float().norm(dim=dims, keepdim=True)
        maxn = clip * wn
        scale = torch.where(gn > maxn, maxn / (gn + 1e-6), torch.ones_like(gn))
        p.grad.mul_(scale.to(p.grad.dtype))


__all__ = ["StepInfo", "Optimizer", "Adam", "AdamW", "SGD", "Adamax", "NAdam", "Nadam", "RAdam", "Lamb", "Lion",
           "NovoGrad", "RMSprop", "Adagrad", "Adadelta", "Adafactor", "Adan", "Sophia", "Muon", "SAM",
           "Lookahead", "EMA", "SWA", "clip_grad_norm_", "clip_grad_value_", "adaptive_clip_grad_",
           "NonFiniteGradient"]
