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

    def load_balance_loss(self, valid_len: torch.Tensor | None = None) -> torch.Tensor:
        """``valid_len`` (a device scalar, an extension): only the first ``valid_len``
        positions of the last scores count, as if the rest did not exist -- the
        escalation path runs Tier 2 on fixed-capacity buffers whose trailing slots
        the reference never creates."""
        if self._last_scores is None:
            return torch.tensor(0.0)
        s = self._last_scores
        if valid_len is not None:
            return self._masked_balance(s, valid_len)
        # var() of a single value is NaN (the reference returns NaN for batch 1
        # or a single chunk); a lone value has zero spread, so it contributes 0.
        chunk_load, per_sample = s.mean(dim=0).float(), s.mean(dim=-1).float()
        loss = chunk_load.var() if chunk_load.numel() > 1 else chunk_load.sum() * 0
        return loss + (per_sample.var() if per_sample.numel() > 1 else per_sample.sum() * 0)

    @staticmethod
    def _masked_balance(s: torch.Tensor, valid_len: torch.Tensor) -> torch.Tensor:
        """The balance loss over positions ``[0, valid_len)`` of ``s (B, P)`` with the
        count on the device: unbiased variances written out with masked sums."""
        s = s.float()
        B, P = s.shape
        m = (torch.arange(P, device=s.device) < valid_len).float()  # (P,)
        n = m.sum()
        chunk_load = s.mean(dim=0)  # (P,)
        mu = (chunk_load * m).sum() / n
        var_c = (((chunk_load - mu) ** 2) * m).sum() / (n - 1).clamp_min(1)
        var_c = torch.where(n > 1, var_c, torch.zeros_like(var_c))
        per_sample = (s * m).sum(dim=1) / n  # (B,)
        var_s = per_sample.var() if B > 1 else per_sample.sum() * 0
        return var_c + var_s
