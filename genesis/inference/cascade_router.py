"""Inference-time tier routing statistics (``genesis/inference/cascade_router.py:15-170``).

:class:`CascadeStats` counts tokens that reached each tier; the compute model
charges Tier 1 = 1, Tier 2 = 3, Tier 3 = 5 units per token.
:class:`CascadeRouter` applies (optionally overridden) gate thresholds.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

TIER_COST = (1, 3, 5)


@dataclass
class CascadeStats:
    tier1_tokens: int = 0
    tier2_tokens: int = 0
    tier3_tokens: int = 0
    total_tokens: int = 0

    def update(self, num_tokens: int, tier2_activated: bool, tier3_activated: bool) -> None:
        self.total_tokens += num_tokens
        self.tier1_tokens += num_tokens
        self.tier2_tokens += num_tokens if tier2_activated else 0
        self.tier3_tokens += num_tokens if tier3_activated else 0

    @property
    def tier1_rate(self) -> float:
        return 1.0

    @property
    def tier2_rate(self) -> float:
        return self.tier2_tokens / self.total_tokens if self.total_tokens else 0.0

    @property
    def tier3_rate(self) -> float:
        return self.tier3_tokens / self.total_tokens if self.total_tokens else 0.0

    @property
    def compute_savings(self) -> float:
        if not self.total_tokens:
            return 0.0
        full = self.total_tokens * sum(TIER_COST)
        used = self.tier1_tokens * TIER_COST[0] + self.tier2_tokens * TIER_COST[1] + self.tier3_tokens * TIER_COST[2]
        return 1.0 - used / full

    def reset(self) -> None:
        self.tier1_tokens = self.tier2_tokens = self.tier3_tokens = self.total_tokens = 0

    def summary(self) -> str:
        return (f"Cascade Stats: {self.total_tokens} tokens | T1: 100% | T2: {self.tier2_rate:.1%} | "
                f"T3: {self.tier3_rate:.1%} | Savings: {self.compute_savings:.1%}")


class CascadeRouter:
    def __init__(self, gate1_threshold: float | None = None, gate2_threshold: float | None = None) -> None:
        self.gate1_threshold = gate1_threshold
        self.gate2_threshold = gate2_threshold
        self.stats = CascadeStats()

    def should_escalate(self, gate_scores: torch.Tensor, threshold: float):
        mask = gate_scores >= threshold
        return mask, bool(mask.any())

    def route_gate1(self, gate_scores: torch.Tensor, model_threshold: float):
        return self.should_escalate(gate_scores, self.gate1_threshold or model_threshold)

    def route_gate2(self, gate_scores: torch.Tensor, model_threshold: float):
        return self.should_escalate(gate_scores, self.gate2_threshold or model_threshold)

    def record(self, num_tokens: int, tier2_activated: bool, tier3_activated: bool) -> None:
        self.stats.update(num_tokens, tier2_activated, tier3_activated)
