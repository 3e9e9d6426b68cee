"""Chunk-level escalation gate (``genesis/model/tier_gate.py:16-122``).

The sequence is zero-padded to a multiple of ``chunk_size``, mean-pooled per
chunk, passed through ``Linear(d, d/4) -> GELU -> Linear(d/4, 1)`` and a
sigmoid.  Training returns the soft scores as the mask; evaluation returns
``scores >= threshold``.  Balance loss: ``var(mean over batch) + var(mean over
chunks)`` of the scores.  Chunk pooling is one kernel on CUDA
(``llm_research_b200.ops.chunk_mean_pool``).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200 import ops


class TierGate(nn.Module):
    def __init__(self, d_model: int, chunk_size: int = 32, threshold: float = 0.5, eps: float = 1e-6) -> None:
        super().__init__()
        self.d_model = d_model
        self.chunk_size = chunk_size
        self.threshold = threshold
        self.eps = eps
        hidden = max(d_model // 4, 1)
        self.gate_mlp = nn.Sequential(nn.Linear(d_model, hidden), nn.GELU(), nn.Linear(hidden, 1))
        self._last_scores: torch.Tensor | None = None

    def forward(self, x: torch.Tensor):
        S = x.shape[1]
        pad = (-S) % self.chunk_size
        if pad:
            x = F.pad(x, (0, 0, 0, pad))
        pooled = ops.chunk_mean_pool(x, self.chunk_size)
        scores = torch.sigmoid(self.gate_mlp(pooled).squeeze(-1))
        self._last_scores = scores
        mask = scores if self.training else scores >= self.threshold
        return mask, scores

    def load_balance_loss(self) -> torch.Tensor:
        if self._last_scores is None:
            return torch.tensor(0.0)
        s = self._last_scores
        # var() of a single value is NaN (the reference returns NaN for batch 1
        # or a single chunk); a lone value has zero spread, so it contributes 0.
        chunk_load, per_sample = s.mean(dim=0).float(), s.mean(dim=-1).float()
        loss = chunk_load.var() if chunk_load.numel() > 1 else chunk_load.sum() * 0
        return loss + (per_sample.var() if per_sample.numel() > 1 else per_sample.sum() * 0)
