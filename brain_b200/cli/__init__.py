"""Command line interface (python -m brain_b200 <command>)."""
from .main import main  # noqa: F401
