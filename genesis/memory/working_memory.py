"""Level-1 working memory: typed slots, gated write, relevance decay
(``genesis/memory/working_memory.py:23-237``).

State ``memory_slots (S, d)`` and ``type_vectors (S, d_type)`` (gradient-linked
through StateLink).  One ``forward``:

1. read: cross-attention from the hidden states to the slots; fuse with a
   sigmoid gate over ``[h, read]``;
2. write: batch/sequence mean -> sigmoid write gate x content, softmax slot
   weights, convex blend ``slots = (1 - w) slots + w * content``; type
   vectors = softmax(type logits) @ type embeddings;
3. erase: slots whose learned relevance is below 0.1 are scaled by
   ``relevance / 0.1``;
4. output ``LayerNorm(aug + out_proj(aug))``.
``utilization_loss = 1 - H(softmax(||slot||)) / log S``.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from genesis.memory.memory_cross_attention import MemoryCrossAttention
from olympus.core.stateful_module import StatefulModule


class WorkingMemory(StatefulModule):
    TYPE_NAMES = ("entity", "relation", "quantity", "temporal", "spatial")

    def __init__(self, num_slots: int = 256, d_model: int = 768, d_type: int = 32, num_types: int = 5,
                 num_heads: int = 8) -> None:
        super().__init__()
        self.num_slots = num_slots
        self.d_model = d_model
        self.d_type = d_type
        self.num_types = num_types
        self.register_state("memory_slots", torch.zeros(num_slots, d_model))
        self.register_state("type_vectors", torch.zeros(num_slots, d_type))
        self.type_embeddings = nn.Embedding(num_types, d_type)
        self.slot_type_logits = nn.Parameter(torch.randn(num_slots, num_types) * 0.02)
        self.read_attn = MemoryCrossAttention(d_model=d_model, num_heads=num_heads, d_memory=d_model)
        self.read_gate = nn.Sequential(nn.Linear(2 * d_model, d_model), nn.Sigmoid())
        self.write_gate_proj = nn.Linear(d_model, d_model)
        self.write_content_proj = nn.Linear(d_model, d_model)
        self.slot_selector = nn.Linear(d_model, num_slots)
        self.relevance_proj = nn.Sequential(nn.Linear(d_model, d_model // 4), nn.ReLU(), nn.Linear(d_model // 4, 1),
                                            nn.Sigmoid())
        self.out_proj = nn.Linear(d_model, d_model)
        self.layer_norm = nn.LayerNorm(d_model)

    def read(self, hidden_states: torch.Tensor) -> torch.Tensor:
        slots = self.link_state("memory_slots").to(hidden_states.dtype)
        return self.read_attn(hidden_states, slots, slots)

    def write(self, hidden_states: torch.Tensor) -> None:
        slots = self.link_state("memory_slots")
        h = hidden_states.mean(dim=(0, 1)).to(slots.dtype)
        content = torch.sigmoid(self.write_gate_proj(h)) * self.write_content_proj(h)
        w = torch.softmax(self.slot_selector(h), dim=0)[:, None]
        self.set_state("memory_slots", (1 - w) * slots + w * content[None])
        types = torch.softmax(self.slot_type_logits, dim=-1) @ self.type_embeddings.weight
        self.set_state("type_vectors", types)

    def erase(self, relevance_threshold: float = 0.1) -> None:
        slots = self.link_state("memory_slots")
        rel = self.relevance_proj(slots).squeeze(-1)
        decay = torch.where(rel > relevance_threshold, torch.ones_like(rel), rel / relevance_threshold)
        self.set_state("memory_slots", slots * decay[:, None])

    def utilization_loss(self) -> torch.Tensor:
        slots = self.get_state("memory_slots")
        p = F.softmax(slots.norm(dim=-1), dim=0)
        ent = -(p * torch.log(p + 1e-8)).sum()
        return 1.0 - ent / torch.log(torch.tensor(float(self.num_slots), device=slots.device))

    def forward(self, hidden_states: torch.Tensor, context: Optional[dict] = None) -> torch.Tensor:
        read_out = self.read(hidden_states)
        gate = self.read_gate(torch.cat([hidden_states, read_out], dim=-1))
        aug = hidden_states + gate * read_out
        self.write(hidden_states)
        self.erase()
        return self.layer_norm(aug + self.out_proj(aug))
