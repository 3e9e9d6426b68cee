"""PHMA semantic-memory read inside the Tier-1 trunk (an extension: the
reference's PHMA stack, ``genesis/memory/semantic_memory.py:22-259``, is not
wired into HLRT).

``MemoryBank``: one store shared by every memory layer -- ``keys (slots, d_key)``
and ``values (slots, d_value)`` buffers (bf16), keys kept L2-normalised so the
cosine read of the semantic memory is a dot product.

``MemoryReadLayer`` (after every ``every``-th block), following
``SemanticMemory.forward`` (``semantic_memory.py:136-146``) as a residual
branch: ``h = RMSNorm(x)``; ``r = W_v read(W_q h)`` with the read = softmax
over the top-k cosine similarities weighting their values; ``x + sigmoid(W_g
[h; r]) * r``.  The read runs on the fused similarity + streaming top-32
kernels (``llm_research_b200.ops.memory.bank_read``); the bank receives no
gradient (it is memory state, written through ``MemoryBank.write``).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from genesis.model.rmsnorm import RMSNorm
from llm_research_b200.ops.linear import project
from llm_research_b200.ops.memory import bank_read


class MemoryBank(nn.Module):
    def __init__(self, slots: int, d_key: int, d_value: int, dtype=torch.bfloat16) -> None:
        super().__init__()
        self.slots, self.d_key, self.d_value = slots, d_key, d_value
        self.register_buffer("keys", F.normalize(torch.randn(slots, d_key), dim=-1).to(dtype))
        self.register_buffer("values", (torch.randn(slots, d_value) * 0.02).to(dtype))
        self.register_buffer("num_written", torch.zeros(1, dtype=torch.long))

    @torch.no_grad()
    def write(self, key: torch.Tensor, value: torch.Tensor) -> None:
        """FIFO ring write of ``(n, d_key)`` keys (normalised here) and their values."""
        key = F.normalize(key.reshape(-1, self.d_key).float(), dim=-1)
        value = value.reshape(-1, self.d_value)
        n = int(self.num_written)
        idx = (n + torch.arange(key.shape[0], device=self.keys.device)) % self.slots
        self.keys[idx] = key.to(self.keys.dtype)
        self.values[idx] = value.to(self.values.dtype)
        self.num_written.add_(key.shape[0])

    def read(self, q: torch.Tensor, top_k: int) -> torch.Tensor:
        out, _ = bank_read(q, self.keys, self.values, top_k)
        return out


class MemoryReadLayer(nn.Module):
    def __init__(self, d_model: int, d_key: int, d_value: int, top_k: int = 32, norm_eps: float = 1e-6) -> None:
        super().__init__()
        from llm_research_b200.parallel.tp import current_tensor_parallel

        self.top_k = top_k
        self.norm = RMSNorm(d_model, eps=norm_eps)
        self.query_proj = nn.Linear(d_model, d_key, bias=False)
        self.value_proj = nn.Linear(d_value, d_model, bias=False)
        self.gate_proj = nn.Linear(2 * d_model, d_model, bias=False)
        self.tp = current_tensor_parallel()  # under TP: runs on sequence shards with replicated weights
        self._bank: Optional[MemoryBank] = None  # shared; not a submodule (saved once, by the model)

    def bind(self, bank: MemoryBank) -> "MemoryReadLayer":
        object.__setattr__(self, "_bank", bank)
        return self

    def _w(self, p: torch.Tensor) -> torch.Tensor:
        if self.tp is None:
            return p
        from llm_research_b200.parallel.tp import sum_grad

        return sum_grad(p, self.tp[0])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from llm_research_b200 import ops

        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        h = ops.rms_norm(x2, self._w(self.norm.weight), self.norm.eps)
        q = project(h, self._w(self.query_proj.weight))
        r = project(self._bank.read(q, self.top_k).to(h.dtype), self._w(self.value_proj.weight))
        g = torch.sigmoid(project(torch.cat([h, r], dim=-1), self._w(self.gate_proj.weight)))
        return (x2 + g * r).view(shape)
