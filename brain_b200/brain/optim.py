"""``brain.optim``: SGD, Adam and AdamW over ``Value`` parameters (reference python/brain/optim and
crates/brain-python/src/optim.rs), stepping with this framework's optimizers (reference AdamW order:
decoupled decay before the moment update). ``zero_grad`` resets every gradient to ``None``."""
from __future__ import annotations

from ..optim import optimizers as _O


class _Wrapped:
    _cls = None

    def __init__(self, params, **kw):
        self.params = list(params)
        self._opt = self._cls([p._t for p in self.params], **kw)

    def step(self) -> None:
        self._opt.step()

    def zero_grad(self) -> None:
        for p in self.params:
            p.zero_grad()

    @property
    def lr(self) -> float:
        return self._opt.get_lr()

    @lr.setter
    def lr(self, v: float) -> None:
        self._opt.set_lr(v)


class SGD(_Wrapped):
    _cls = _O.SGD

    def __init__(self, params, lr: float = 0.01, momentum: float = 0.0, weight_decay: float = 0.0):
        super().__init__(params, lr=lr, momentum=momentum, weight_decay=weight_decay)


class Adam(_Wrapped):
    _cls = _O.Adam

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.0):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)


class AdamW(_Wrapped):
    _cls = _O.AdamW

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.01):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)


__all__ = ["SGD", "Adam", "AdamW"]
