"""Checkpoint formats (reference-compatible .brain text / binary / archive / .bn, and BRAINCK2)."""
from .formats import *  # noqa: F401,F403
from .formats import ModelState, TensorArchive, BrainModelFile, save_brain_v2, load_brain_v2  # noqa: F401
