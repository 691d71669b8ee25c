"""Distributed runtime: process groups, collectives, data/tensor/pipeline parallel engines."""
from . import dist  # noqa: F401
from .dist import DistributedContext, ProcessGroup, init, barrier, shutdown, rank_prefix  # noqa: F401
from .flat import FlatParams  # noqa: F401
from .ddp import DataParallel  # noqa: F401
