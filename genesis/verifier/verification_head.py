"""Multi-task verification heads (``genesis/verifier/verification_head.py:17-154``).

Four ``sigmoid(Linear(d, 1))`` scores (factual, logical, stylistic, overall),
computed as ONE ``(d → 4)`` projection; the four sub-modules keep the
reference's parameter names (``factual_head.0.weight`` ...) so checkpoints
interchange.  ``compute_loss`` sums per-head BCE; a missing overall label is
``0.4·factual + 0.35·logical + 0.25·stylistic``.
"""

from __future__ import annotations

from typing import Dict

import torch
import torch.nn as nn
import torch.nn.functional as F

_KEYS = ("factual_score", "logical_score", "stylistic_score", "overall_score")


class VerificationHead(nn.Module):
    DEFAULT_WEIGHTS: Dict[str, float] = {"factual": 0.4, "logical": 0.35, "stylistic": 0.25}

    def __init__(self, d_model: int = 512) -> None:
        super().__init__()
        self.d_model = d_model
        self.factual_head = nn.Sequential(nn.Linear(d_model, 1), nn.Sigmoid())
        self.logical_head = nn.Sequential(nn.Linear(d_model, 1), nn.Sigmoid())
        self.stylistic_head = nn.Sequential(nn.Linear(d_model, 1), nn.Sigmoid())
        self.overall_head = nn.Sequential(nn.Linear(d_model, 1), nn.Sigmoid())
        for head in self._heads():
            nn.init.xavier_uniform_(head[0].weight)
            nn.init.zeros_(head[0].bias)

    def _heads(self):
        return (self.factual_head, self.logical_head, self.stylistic_head, self.overall_head)

    def forward(self, pooled_hidden: torch.Tensor) -> Dict[str, torch.Tensor]:
        w = torch.cat([h[0].weight for h in self._heads()], dim=0)
        b = torch.cat([h[0].bias for h in self._heads()], dim=0)
        s = torch.sigmoid(F.linear(pooled_hidden, w, b))
        return {k: s[:, i:i + 1] for i, k in enumerate(_KEYS)}

    def compute_loss(self, scores: Dict[str, torch.Tensor], labels: Dict[str, torch.Tensor]) -> torch.Tensor:
        ref = scores["overall_score"]
        loss = torch.zeros((), device=ref.device, dtype=ref.dtype)
        for key in _KEYS[:3]:
            if key in labels:
                loss = loss + F.binary_cross_entropy(scores[key], labels[key].to(scores[key].dtype))
        if "overall_score" in labels:
            target = labels["overall_score"]
        else:
            zero = torch.zeros_like(ref)
            target = (self.DEFAULT_WEIGHTS["factual"] * labels.get("factual_score", zero)
                      + self.DEFAULT_WEIGHTS["logical"] * labels.get("logical_score", zero)
                      + self.DEFAULT_WEIGHTS["stylistic"] * labels.get("stylistic_score", zero))
        return loss + F.binary_cross_entropy(ref, target.to(ref.dtype))
