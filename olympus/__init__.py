"""Olympus: a training runtime for stateful, multi-model training on B200 (sm_100a)."""
from olympus.version import __version__

__all__ = ["__version__"]
