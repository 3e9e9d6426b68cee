"""Mixture-of-experts SwiGLU FFN (``genesis/model/moe.py:17-109``).

``y[n] = sum_k w[n,k] * expert_{idx[n,k]}(x[n])``.  The reference loops over
``(k, expert)`` with boolean masks (one host sync each).  Here tokens are
grouped by expert with one sort and each expert runs once on its contiguous
slice (one host read of the per-expert counts per layer).

``capacity_factor``: the reference stores it without using it.  With
``enforce_capacity=True`` each expert keeps at most
``ceil(capacity_factor * N * top_k / E)`` assignments (lowest token index
first) and drops the rest, which is the capacity rule the expert-parallel
path (``llm_research_b200.parallel.expert_parallel``) uses.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from genesis.model.ffn import SwiGLUFFN
from genesis.model.moe_router import ExpertRouter
from olympus.core.compute_router import grouped_expert_apply


def capacity_mask(indices: torch.Tensor, num_experts: int, capacity: int) -> torch.Tensor:
    """Bool ``(N, k)``: True where the assignment fits in its expert's capacity.

    Assignments are ranked per expert in (token, k) order.
    """
    flat = indices.reshape(-1)
    onehot = torch.nn.functional.one_hot(flat, num_experts)
    rank = (onehot.cumsum(0) * onehot).sum(-1) - 1
    return (rank < capacity).reshape(indices.shape)


class MoEFFN(nn.Module):
    def __init__(
        self,
        d_model: int,
        d_ff: int | None = None,
        num_experts: int = 8,
        top_k: int = 2,
        capacity_factor: float = 1.25,
        dropout: float = 0.0,
        jitter_noise: float = 0.0,
        enforce_capacity: bool = False,
        num_shared_experts: int = 0,
    ) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_experts = num_experts
        self.top_k = top_k
        self.capacity_factor = capacity_factor
        self.enforce_capacity = enforce_capacity
        self.router = ExpertRouter(d_model=d_model, num_experts=num_experts, top_k=top_k, jitter_noise=jitter_noise)
        self.experts = nn.ModuleList([SwiGLUFFN(d_model=d_model, d_ff=d_ff, dropout=dropout) for _ in range(num_experts)])
        # always-on experts added to every token (DeepSeek-style shared experts); none in the reference
        self.shared_experts = nn.ModuleList([SwiGLUFFN(d_model=d_model, d_ff=d_ff, dropout=dropout)
                                             for _ in range(num_shared_experts)])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        xf = x.reshape(-1, shape[-1])
        w, idx, _ = self.router(xf)
        if self.enforce_capacity:
            cap = math.ceil(self.capacity_factor * xf.shape[0] * self.top_k / self.num_experts)
            w = w * capacity_mask(idx, self.num_experts, cap).to(w.dtype)
        out = grouped_expert_apply(xf, idx, w, self.experts, self.num_experts)
        for e in self.shared_experts:
            out = out + e(xf)
        return out.to(x.dtype).reshape(shape)

    def load_balance_loss(self) -> torch.Tensor:
        return self.router.load_balance_loss()
