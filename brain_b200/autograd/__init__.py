"""Autograd API of the reference (Value, Tape, no_grad, functional transforms, GradScaler)."""
from .value import (Value, NoGradGuard, no_grad, with_no_grad, is_grad_enabled, backward_from,  # noqa: F401
                    backward_with_grad, set_grad_enabled, with_enable_grad, grad_of, zero_grad_from)
from .tape import Tape, OpRecord, start_recording, stop_recording, with_tape, is_recording, TapePruner, TapeFusionPass  # noqa: F401
from .functional import (grad, value_and_grad, vjp, jvp, jacobian, hessian, grad_and_hess, numeric_grad,  # noqa: F401
                         checkpoint, BudgetCheckpoint, CheckpointPolicy, CpuOffloader, GradScaler,
                         parallel_backward)
from .graph import topological_sort, compute_dag_levels, values_close, TapeBuilder, RecomputeGraph  # noqa: F401
from . import vjps  # noqa: F401
from .vjps import unbroadcast  # noqa: F401
