"""Reproducibility (``olympus/utils/seeds.py:16-36``)."""

from __future__ import annotations

import random

import torch

try:
    import numpy as np

    _HAS_NUMPY = True
except ImportError:  # pragma: no cover
    _HAS_NUMPY = False


def set_seed(seed: int = 42, deterministic_cudnn: bool = True) -> None:
    """Seed python, numpy, torch (CPU and every CUDA device); optionally make cuDNN deterministic."""
    random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    if _HAS_NUMPY:
        np.random.seed(seed)
    if deterministic_cudnn and torch.cuda.is_available():
        torch.backends.cudnn.deterministic = True
        torch.backends.cudnn.benchmark = False
