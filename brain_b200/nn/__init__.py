"""Neural-network layers with the reference's names (brain-nn), on the sm_100a ops."""
from .module import Module, Sequential, ModuleList, ModuleDict, Identity  # noqa: F401
from .layers import *  # noqa: F401,F403
from . import init  # noqa: F401
