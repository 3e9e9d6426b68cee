"""Level-2 episodic memory: surprise-gated ring-buffer writes
(``genesis/memory/episodic_memory.py:27-278``).

State: ``episodic_slots (S, d)``, ``slot_ages (S)``, ``write_pointer (1)``,
``running_loss_mean/var (1)`` (EMA, momentum 0.01).  A token is *surprising*
when its loss z-score exceeds ``importance_threshold``; the surprising tokens
of each sequence are pooled with learned importance weights into one
``write_proj`` vector written to the next ring slot.  The batch mean of the
writes is published on the memory bus (``episodic_context``, scope
``episode``) and concatenated to the slots when reading, which shares
episodes across sequences.

The ring write is one indexed copy (the reference loops over the batch) and
the surprise statistics stay on the device.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from genesis.memory.memory_cross_attention import MemoryCrossAttention
from olympus.core.memory_bus import MemoryBus
from olympus.core.stateful_module import StatefulModule


class EpisodicMemory(StatefulModule):
    def __init__(self, num_slots: int = 1024, d_model: int = 768, num_heads: int = 8,
                 importance_threshold: float = 1.5, memory_bus: Optional[MemoryBus] = None) -> None:
        super().__init__()
        self.num_slots = num_slots
        self.d_model = d_model
        self.importance_threshold = importance_threshold
        self.memory_bus = memory_bus if memory_bus is not None else MemoryBus()
        self.register_state("episodic_slots", torch.zeros(num_slots, d_model))
        self.register_state("slot_ages", torch.zeros(num_slots))
        self.register_state("write_pointer", torch.zeros(1, dtype=torch.long))
        self.register_state("running_loss_mean", torch.ones(1))
        self.register_state("running_loss_var", torch.ones(1))
        self.read_attn = MemoryCrossAttention(d_model=d_model, num_heads=num_heads, d_memory=d_model)
        self.read_gate = nn.Sequential(nn.Linear(2 * d_model, d_model), nn.Sigmoid())
        self.importance_scorer = nn.Sequential(nn.Linear(d_model + 1, d_model // 4), nn.ReLU(),
                                               nn.Linear(d_model // 4, 1), nn.Sigmoid())
        self.write_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)
        self.layer_norm = nn.LayerNorm(d_model)

    def _compute_surprise(self, loss_per_token: torch.Tensor) -> torch.Tensor:
        mean = self.get_state("running_loss_mean")
        std = self.get_state("running_loss_var").clamp(min=1e-12).sqrt().clamp(min=1e-6)
        return ((loss_per_token - mean) / std).clamp(min=0.0)

    def _update_loss_statistics(self, loss_per_token: torch.Tensor, momentum: float = 0.01) -> None:
        m = loss_per_token.detach().float().mean()
        v = loss_per_token.detach().float().var().clamp(min=1e-6)
        self.set_state("running_loss_mean", (1 - momentum) * self.get_state("running_loss_mean") + momentum * m)
        self.set_state("running_loss_var", (1 - momentum) * self.get_state("running_loss_var") + momentum * v)

    def read(self, query: torch.Tensor) -> torch.Tensor:
        keys = self.link_state("episodic_slots")
        bus = self.memory_bus.read("episodic_context", scope="episode")
        if bus is not None and bus.dim() == 2 and bus.size(-1) == self.d_model:
            keys = torch.cat([keys, bus.to(keys.device, keys.dtype)], dim=0)
        keys = keys.to(query.dtype)
        return self.read_attn(query, keys, keys)

    def write_if_important(self, hidden_states: torch.Tensor, loss_per_token: torch.Tensor) -> None:
        self._update_loss_statistics(loss_per_token)
        mask = self._compute_surprise(loss_per_token) > self.importance_threshold
        if not bool(mask.any()):
            return
        feats = torch.cat([hidden_states, loss_per_token.unsqueeze(-1).to(hidden_states.dtype)], dim=-1)
        w = self.importance_scorer(feats).squeeze(-1) * mask.to(hidden_states.dtype)
        pooled = (w.unsqueeze(-1) * hidden_states).sum(1) / w.sum(1, keepdim=True).clamp(min=1e-8)
        content = self.write_proj(pooled).detach()
        B = content.shape[0]
        ptr = self.get_state("write_pointer")
        slots = self.get_state("episodic_slots").clone()
        ages = self.get_state("slot_ages").clone()
        idx = (ptr + torch.arange(B, device=ptr.device)) % self.num_slots
        slots[idx] = content.to(slots.dtype)
        ages[idx] = 0.0
        self.set_state("episodic_slots", slots)
        self.set_state("write_pointer", (ptr + B) % self.num_slots)
        self.set_state("slot_ages", ages + 1.0)
        self.memory_bus.write("episodic_context", content.mean(dim=0, keepdim=True), scope="episode")

    def forward(self, hidden_states: torch.Tensor, context: Optional[dict] = None) -> torch.Tensor:
        read_out = self.read(hidden_states)
        aug = hidden_states + self.read_gate(torch.cat([hidden_states, read_out], dim=-1)) * read_out
        if context is not None and "loss_per_token" in context:
            self.write_if_important(hidden_states, context["loss_per_token"])
        return self.layer_norm(aug + self.out_proj(aug))
