"""Level-3 semantic memory: key/value store with top-k cosine retrieval
(``genesis/memory/semantic_memory.py:22-259``).

Buffers ``keys (N, d_key)``, ``values (N, d_value)``, ``num_written``,
``_frozen``.  ``read(q)``: cosine similarity of each query against the
populated keys, top-k, softmax over the k similarities, weighted sum of the
k values.  Writes fill a FIFO ring; frozen stores reject writes.

On CUDA the read is the fused top-k memory kernel
(``llm_research_b200.ops.memory.topk_memory_read``): similarity tiles,
per-query streaming top-k and the value gather in one pass, without
materialising the ``(queries, N)`` similarity matrix.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200.ops.memory import topk_memory_read


class SemanticMemory(nn.Module):
    def __init__(self, num_entries: int = 10000, d_key: int = 256, d_value: int = 768, d_model: int = 768,
                 top_k: int = 5) -> None:
        super().__init__()
        self.num_entries = num_entries
        self.d_key = d_key
        self.d_value = d_value
        self.d_model = d_model
        self.default_top_k = top_k
        self.register_buffer("keys", torch.zeros(num_entries, d_key))
        self.register_buffer("values", torch.zeros(num_entries, d_value))
        self.register_buffer("num_written", torch.zeros(1, dtype=torch.long))
        self.register_buffer("_frozen", torch.zeros(1, dtype=torch.bool))
        self.query_proj = nn.Linear(d_model, d_key)
        self.value_proj = nn.Linear(d_value, d_model)
        self.output_gate = nn.Sequential(nn.Linear(2 * d_model, d_model), nn.Sigmoid())
        self.layer_norm = nn.LayerNorm(d_model)
        nn.init.normal_(self.keys, std=0.02)

    def read(self, query: torch.Tensor, top_k: Optional[int] = None) -> torch.Tensor:
        k = self.default_top_k if top_k is None else top_k
        n = int(self.num_written)
        if n == 0:
            return torch.zeros(*query.shape[:-1], self.d_value, device=query.device, dtype=query.dtype)
        q = query.reshape(-1, self.d_key)
        out = topk_memory_read(q, self.keys[:n], self.values[:n], min(k, n))
        return out.reshape(*query.shape[:-1], self.d_value).to(query.dtype)

    @torch.no_grad()
    def write(self, key: torch.Tensor, value: torch.Tensor) -> None:
        if bool(self._frozen):
            raise RuntimeError("SemanticMemory is frozen; writes are not allowed.")
        key = key.reshape(-1, self.d_key)
        value = value.reshape(-1, self.d_value)
        n = int(self.num_written)
        idx = (n + torch.arange(key.shape[0], device=self.keys.device)) % self.num_entries
        self.keys[idx] = key.detach().to(self.keys.dtype)
        self.values[idx] = value.detach().to(self.values.dtype)
        self.num_written.fill_(min(n + key.shape[0], self.num_entries))

    @torch.no_grad()
    def update(self, key_idx: int, new_value: torch.Tensor) -> None:
        if bool(self._frozen):
            raise RuntimeError("SemanticMemory is frozen; updates are not allowed.")
        n = int(self.num_written)
        if key_idx < 0 or key_idx >= n:
            raise IndexError(f"key_idx {key_idx} out of range for {n} written entries.")
        self.values[key_idx] = new_value.detach().to(self.values.dtype)

    def freeze(self) -> None:
        self._frozen.fill_(True)

    def unfreeze(self) -> None:
        self._frozen.fill_(False)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        retrieved = self.value_proj(self.read(self.query_proj(hidden_states)))
        gate = self.output_gate(torch.cat([hidden_states, retrieved], dim=-1))
        return self.layer_norm(hidden_states + gate * retrieved)

    def retrieval_loss(self, query: torch.Tensor, expected_value: torch.Tensor) -> torch.Tensor:
        return F.mse_loss(self.read(query), expected_value)
