"""Generic top-k expert router (``olympus/core/compute_router.py:22-257``).

``plan`` maps tokens to a :class:`RoutePlan` (softmax -> top-k -> renormalise);
``execute`` runs arbitrary expert modules on their tokens and combines the
outputs with the routing weights.  Gates: ``linear``, ``mlp`` (Linear-ReLU-
Linear) and ``entropy`` (linear gate plus an entropy bonus in the balance loss).

Execution groups tokens by expert with one stable sort and one host read of
the per-expert counts, instead of one boolean mask (and one sync) per
``(k, expert)`` pair; the combination is the same weighted sum.

The reference computes a straight-through mask during training whose value
is discarded (its forward is unchanged by it); that no-op is not reproduced.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Literal, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class RoutePlan:
    expert_indices: torch.Tensor  # (N, top_k) int64
    expert_weights: torch.Tensor  # (N, top_k) rows sum to 1
    raw_logits: torch.Tensor      # (N, E)
    probabilities: torch.Tensor   # (N, E)

    @property
    def num_experts(self) -> int:
        return int(self.probabilities.shape[-1])

    @property
    def top_k(self) -> int:
        return int(self.expert_indices.shape[-1])


def grouped_expert_apply(
    x_flat: torch.Tensor,
    indices: torch.Tensor,
    weights: torch.Tensor,
    experts,
    num_experts: int,
) -> torch.Tensor:
    """``sum_k w[n,k] * experts[idx[n,k]](x[n])`` with tokens grouped per expert."""
    n_tok, top_k = indices.shape
    flat_e = indices.reshape(-1)
    order = torch.argsort(flat_e, stable=True)
    token_of = order // top_k
    counts = torch.bincount(flat_e, minlength=num_experts).tolist()
    xs = x_flat.index_select(0, token_of)
    w = weights.reshape(-1).index_select(0, order).unsqueeze(-1)
    pieces = []
    start = 0
    for e, c in enumerate(counts):
        if c:
            pieces.append(experts[e](xs[start:start + c]))
        start += c
    if not pieces:
        return torch.zeros_like(x_flat)
    ys = torch.cat(pieces, 0) * w.to(pieces[0].dtype)
    out = torch.zeros(n_tok, ys.shape[-1], dtype=ys.dtype, device=ys.device)
    return out.index_add(0, token_of, ys)


class ComputeRouter(nn.Module):
    def __init__(
        self,
        input_dim: int,
        num_experts: int,
        top_k: int = 2,
        gate_type: Literal["linear", "mlp", "entropy"] = "linear",
        gate_hidden: int = 128,
        entropy_coeff: float = 0.01,
        load_balance_coeff: float = 0.01,
    ) -> None:
        super().__init__()
        if gate_type not in ("linear", "mlp", "entropy"):
            raise ValueError(f"Unknown gate_type '{gate_type}'. Use 'linear', 'mlp', or 'entropy'.")
        self.input_dim = input_dim
        self.num_experts = num_experts
        self.top_k = min(top_k, num_experts)
        self.gate_type = gate_type
        self.entropy_coeff = entropy_coeff
        self.load_balance_coeff = load_balance_coeff
        if gate_type == "mlp":
            self.gate = nn.Sequential(nn.Linear(input_dim, gate_hidden), nn.ReLU(), nn.Linear(gate_hidden, num_experts))
        else:
            self.gate = nn.Linear(input_dim, num_experts, bias=False)
        self.reset_stats()

    @staticmethod
    def _flatten(x: torch.Tensor) -> torch.Tensor:
        if x.dim() == 3:
            return x.reshape(-1, x.shape[-1])
        if x.dim() == 2:
            return x
        raise ValueError(f"Expected 2-D or 3-D input, got {x.dim()}-D.")

    def plan(self, x: torch.Tensor) -> RoutePlan:
        xf = self._flatten(x)
        logits = self.gate(xf)
        probs = F.softmax(logits, dim=-1)
        w, idx = torch.topk(probs, self.top_k, dim=-1)
        w = w / (w.sum(dim=-1, keepdim=True) + 1e-9)
        with torch.no_grad():
            self._total_tokens += xf.shape[0]
            self._total_steps += 1
            hist = torch.bincount(idx.reshape(-1), minlength=self.num_experts).to(torch.float32)
            self._expert_counts = self._expert_counts.to(hist.device) + hist
        return RoutePlan(expert_indices=idx, expert_weights=w, raw_logits=logits, probabilities=probs)

    def execute(self, x: torch.Tensor, experts: nn.ModuleList, route_plan: Optional[RoutePlan] = None) -> torch.Tensor:
        plan = route_plan if route_plan is not None else self.plan(x)
        xf = self._flatten(x)
        out = grouped_expert_apply(xf, plan.expert_indices, plan.expert_weights, experts, self.num_experts)
        return out.reshape(*x.shape[:-1], out.shape[-1]).to(x.dtype)

    def load_balance_loss(self, route_plan: RoutePlan) -> torch.Tensor:
        """Switch-style ``coeff * E * sum_i f_i P_i`` (minus an entropy bonus for ``entropy``)."""
        probs = route_plan.probabilities
        n = probs.shape[0]
        e = self.num_experts
        counts = F.one_hot(route_plan.expert_indices, num_classes=e).float().sum(dim=(0, 1))
        frac = counts / (n * self.top_k + 1e-9)
        loss = self.load_balance_coeff * e * (frac * probs.mean(dim=0)).sum()
        if self.gate_type == "entropy":
            ent = -(probs * (probs + 1e-9).log()).sum(dim=-1).mean()
            loss = loss - self.entropy_coeff * ent
        return loss

    def get_routing_stats(self) -> Dict[str, object]:
        if self._total_tokens == 0:
            return {"total_tokens": 0, "total_steps": 0}
        counts = self._expert_counts.float().cpu()
        frac = counts / (counts.sum() + 1e-9)
        uniform = 1.0 / self.num_experts + 1e-9
        return {
            "total_tokens": self._total_tokens,
            "total_steps": self._total_steps,
            "expert_utilization": {f"expert_{i}": float(frac[i]) for i in range(self.num_experts)},
            "max_load_ratio": float(frac.max()) / uniform,
            "min_load_ratio": float(frac.min()) / uniform,
        }

    def reset_stats(self) -> None:
        self._total_tokens = 0
        self._total_steps = 0
        self._expert_counts = torch.zeros(self.num_experts)
