"""Top-k expert router with the Switch load-balance loss (``genesis/model/moe_router.py:16-120``).

Optional multiplicative jitter, gate linear, fp32 softmax, top-k,
renormalisation (``w / (sum w + 1e-9)``).  The probabilities and the
per-expert assignment counts are kept for ``E * sum_i f_i * P_i`` (``f_i`` =
count_i / tokens, as the reference's expert mask averaged over tokens).  On
CUDA the gate is the CTA-pair GEMM (``ops.linear.dense``), softmax, top-k and
renormalisation are one kernel (``ops.softmax_topk``) and the counts come from
the routing kernel (``ops.route_slots``), with no host read.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200 import ops


class ExpertRouter(nn.Module):
    def __init__(self, d_model: int, num_experts: int, top_k: int = 2, jitter_noise: float = 0.0) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_experts = num_experts
        self.top_k = top_k
        self.jitter_noise = jitter_noise
        self.gate = nn.Linear(d_model, num_experts, bias=False)
        self._last_router_probs: Optional[torch.Tensor] = None
        self._last_expert_counts: Optional[torch.Tensor] = None

    def forward(self, x: torch.Tensor):
        from llm_research_b200.ops.linear import dense

        if self.training and self.jitter_noise > 0.0:
            x = x * torch.empty_like(x).uniform_(1.0 - self.jitter_noise, 1.0 + self.jitter_noise)
        logits = dense(x, self.gate.weight, self.gate.bias)
        flat = logits.reshape(-1, self.num_experts)
        w, idx, probs = ops.softmax_topk(flat, self.top_k)
        w = w.reshape(*logits.shape[:-1], self.top_k).type_as(x)
        self._last_router_probs = probs
        self._last_expert_counts = ops.route_slots(idx, self.num_experts)[3]
        idx = idx.reshape(*logits.shape[:-1], self.top_k)
        return w, idx, logits

    def load_balance_loss(self) -> torch.Tensor:
        if self._last_router_probs is None or self._last_expert_counts is None:
            return torch.tensor(0.0)
        tokens = max(self._last_router_probs.shape[0], 1)
        f = self._last_expert_counts.float() / tokens
        p = self._last_router_probs.float().mean(dim=0)
        return self.num_experts * (f * p).sum()
