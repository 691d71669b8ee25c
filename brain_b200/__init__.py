"""brain_b200: a B200-native (sm_100a) deep-learning framework with the capabilities of brain.

The reference's Python-package names (``Tensor``, ``Value``, ``zeros``, ``ones``, ``tensor``) are
available here as well as under ``brain_b200.brain`` (with ``brain.nn`` and ``brain.optim``); they are
loaded on first use, so importing the package stays light."""
__version__ = "0.1.0"

_FACADE = ("Tensor", "Value", "zeros", "ones", "tensor")


def __getattr__(name):
    if name in _FACADE:
        from . import brain as _b
        return getattr(_b, name)
    raise AttributeError(f"module 'brain_b200' has no attribute '{name}'")
