"""Contradiction detection between memory entries (``genesis/memory/memory_consistency.py:17-127``).

Entries are compared after a learned projection; a pair is *contradictory*
when its cosine similarity is above ``threshold`` but below 0.99 (near
duplicates are not contradictions).  The loss is the mean excess similarity
over flagged pairs.
"""

from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


class MemoryConsistency(nn.Module):
    def __init__(self, d_model: int, threshold: float = 0.8) -> None:
        super().__init__()
        self.d_model = d_model
        self.threshold = threshold
        self.proj = nn.Linear(d_model, d_model)
        self.layer_norm = nn.LayerNorm(d_model)

    @torch.no_grad()
    def check_consistency(self, new_entry: torch.Tensor, existing_entries: torch.Tensor) -> Tuple[bool, float]:
        if existing_entries.size(0) == 0:
            return False, 0.0
        a = F.normalize(self.proj(new_entry.detach().view(1, -1)), dim=-1)
        b = F.normalize(self.proj(existing_entries.detach()), dim=-1)
        top = float((a @ b.t()).max())
        return (self.threshold < top < 0.99), top

    def consistency_loss(self, memory_writes: torch.Tensor, existing_memory: torch.Tensor) -> torch.Tensor:
        dev = memory_writes.device
        if existing_memory.size(0) == 0 or memory_writes.size(0) == 0:
            return torch.zeros((), device=dev, requires_grad=True)
        a = F.normalize(self.layer_norm(self.proj(memory_writes)), dim=-1)
        b = F.normalize(self.layer_norm(self.proj(existing_memory)), dim=-1)
        sim = a @ b.t()
        flag = (sim > self.threshold) & (sim < 0.99)
        if not bool(flag.any()):
            return torch.zeros((), device=dev, requires_grad=True)
        excess = (sim - self.threshold).clamp(min=0.0) * flag.to(sim.dtype)
        return excess.sum() / flag.to(sim.dtype).sum().clamp(min=1.0)

    def forward(self, new_entries: torch.Tensor, memory_bank: torch.Tensor) -> torch.Tensor:
        return self.consistency_loss(new_entries, memory_bank)
