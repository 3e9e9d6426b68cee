"""Multi-head cross-attention from hidden states to a memory bank
(``genesis/memory/memory_cross_attention.py:17-107``).

Biased q/k/v/o projections; the bank is ``(M, d_mem)`` (shared by the batch)
or ``(B, M, d_mem)``; an optional ``(B, M)`` bool mask marks valid slots.  The
attention itself is :func:`olympus.kernels.memory_cross_attention` (the
flash-attention kernel when there is no mask).
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from olympus.kernels.memory_cross_attention import memory_cross_attention


class MemoryCrossAttention(nn.Module):
    def __init__(self, d_model: int, num_heads: int = 8, d_memory: Optional[int] = None, dropout: float = 0.0) -> None:
        super().__init__()
        assert d_model % num_heads == 0, "d_model must be divisible by num_heads"
        self.d_model = d_model
        self.d_memory = d_memory if d_memory is not None else d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.dropout_p = dropout
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(self.d_memory, d_model)
        self.v_proj = nn.Linear(self.d_memory, d_model)
        self.o_proj = nn.Linear(d_model, d_model)
        self.scale = 1.0 / math.sqrt(self.head_dim)

    def forward(self, query: torch.Tensor, memory_keys: torch.Tensor, memory_values: torch.Tensor,
                memory_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        return memory_cross_attention(query, memory_keys, memory_values, self.q_proj, self.k_proj, self.v_proj,
                                      self.o_proj, self.num_heads, memory_mask=memory_mask,
                                      dropout_p=self.dropout_p, training=self.training)
