"""RMSNorm (``genesis/model/rmsnorm.py:13-49``).

``y = bf(x * rsqrt(mean(x^2) + eps)) * weight`` -- the statistics are taken in
fp32 and the normalised value is rounded to ``x.dtype`` before the weight is
applied, as in the reference.  On CUDA both directions run in one sm_100a
kernel each (``llm_research_b200.ops.rms_norm``).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from llm_research_b200 import ops


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def _norm(self, x: torch.Tensor) -> torch.Tensor:
        return x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + self.eps)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.eps)

    def forward_residual(self, x: torch.Tensor, residual: torch.Tensor):
        """``s = x + residual; return (norm(s), s)`` in one pass."""
        return ops.rms_norm_residual(x, residual, self.weight, self.eps)
