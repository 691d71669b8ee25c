"""Optimizers (brain-optim): fused AdamW / SGD kernels, the reference's optimizer family,
schedulers, clipping, EMA/SWA, and the sharded flat AdamW used by the data-parallel engine."""
from .flat_adamw import FlatAdamW  # noqa: F401
from .optimizers import *  # noqa: F401,F403
from .schedulers import *  # noqa: F401,F403
from ..autograd.functional import GradScaler  # noqa: F401
from .builder import (OptimizerKind, OptimizerBuilder, ParamGroup, ParamGroupConfig, GradEntry,  # noqa: F401
                      Rmsprop, SophiaG, SwAOptimizer, ModelEma, LrFinder, LrScheduler, SgdNesterov)
