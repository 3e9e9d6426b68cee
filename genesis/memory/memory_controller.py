"""Three-level PHMA memory controller (``genesis/memory/memory_controller.py:31-237``).

Runs working, episodic and semantic memory on the hidden states, mixes them
with a per-token softmax gate over ``[work, episodic, semantic]`` (gate EMA
kept as state, momentum 0.99), adds the mix through ``out_proj`` and a
LayerNorm.  In training, each sequence's mean hidden state is written to
semantic memory unless it contradicts an existing value (``MemoryConsistency``).
The contradiction test is batched (one similarity matrix for all sequences)
instead of one check per sequence.
Aux losses: ``utilization`` (working memory), ``consistency`` (last writes vs
episodic slots) and ``retrieval`` (0 without a supervised target).
"""

from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from genesis.memory.episodic_memory import EpisodicMemory
from genesis.memory.memory_consistency import MemoryConsistency
from genesis.memory.semantic_memory import SemanticMemory
from genesis.memory.working_memory import WorkingMemory
from olympus.core.memory_bus import MemoryBus
from olympus.core.stateful_module import StatefulModule


class MemoryController(StatefulModule):
    def __init__(self, d_model: int = 768, num_working_slots: int = 256, num_episodic_slots: int = 1024,
                 num_semantic_entries: int = 10000, d_key: int = 256, num_heads: int = 8,
                 importance_threshold: float = 1.5, consistency_threshold: float = 0.8,
                 memory_bus: Optional[MemoryBus] = None) -> None:
        super().__init__()
        self.d_model = d_model
        self.memory_bus = memory_bus if memory_bus is not None else MemoryBus()
        self.working_memory = WorkingMemory(num_slots=num_working_slots, d_model=d_model, num_heads=num_heads)
        self.episodic_memory = EpisodicMemory(num_slots=num_episodic_slots, d_model=d_model, num_heads=num_heads,
                                              importance_threshold=importance_threshold, memory_bus=self.memory_bus)
        self.semantic_memory = SemanticMemory(num_entries=num_semantic_entries, d_key=d_key, d_value=d_model,
                                              d_model=d_model)
        self.consistency = MemoryConsistency(d_model=d_model, threshold=consistency_threshold)
        self.gate_proj = nn.Linear(3 * d_model, 3)
        self.semantic_key_proj = nn.Linear(d_model, d_key)
        self.semantic_value_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)
        self.layer_norm = nn.LayerNorm(d_model)
        self.register_state("gate_ema", torch.full((3,), 1.0 / 3))
        self._last_write_hidden: Optional[torch.Tensor] = None

    def forward(self, hidden_states: torch.Tensor, context: Optional[dict] = None) -> torch.Tensor:
        outs = [self.working_memory(hidden_states, context=context),
                self.episodic_memory(hidden_states, context=context),
                self.semantic_memory(hidden_states)]
        gates = F.softmax(self.gate_proj(torch.cat(outs, dim=-1)), dim=-1)
        mixed = sum(o * gates[..., i:i + 1] for i, o in enumerate(outs))
        with torch.no_grad():
            self.set_state("gate_ema", 0.99 * self.get_state("gate_ema") + 0.01 * gates.mean(dim=(0, 1)).float())
        if self.training:
            summary = hidden_states.mean(dim=1)
            keys = self.semantic_key_proj(summary)
            vals = self.semantic_value_proj(summary)
            n = int(self.semantic_memory.num_written)
            if n > 0:
                with torch.no_grad():
                    a = F.normalize(self.consistency.proj(vals.detach()), dim=-1)
                    b = F.normalize(self.consistency.proj(self.semantic_memory.values[:n].to(vals.dtype)), dim=-1)
                    top = (a @ b.t()).max(dim=-1).values
                    ok = ~((top > self.consistency.threshold) & (top < 0.99))
                if bool(ok.any()):
                    self.semantic_memory.write(keys[ok], vals[ok])
            else:
                self.semantic_memory.write(keys, vals)
            self._last_write_hidden = vals.detach()
        return self.layer_norm(hidden_states + self.out_proj(mixed))

    def compute_aux_losses(self) -> Dict[str, torch.Tensor]:
        dev = next(self.parameters()).device
        if self._last_write_hidden is not None:
            slots = self.episodic_memory.get_state("episodic_slots").to(self._last_write_hidden.dtype)
            consistency = self.consistency(self._last_write_hidden, slots)
        else:
            consistency = torch.zeros((), device=dev, requires_grad=True)
        return {"utilization": self.working_memory.utilization_loss(), "consistency": consistency,
                "retrieval": torch.zeros((), device=dev, requires_grad=True)}
