"""Progressive model growth (``olympus/core/growth_controller.py:17-210``).

Growth fires either on a schedule of ``(step, event_type, kwargs)`` entries or
adaptively after ``patience`` steps without a loss improvement of
``min_delta`` (adaptive growth is a ``widen`` with ``factor=1.5``).  The tensor
surgery (:meth:`_widen`, :meth:`_deepen`, :meth:`_dense_to_moe`) is model
specific and raises ``NotImplementedError`` here; :class:`genesis.model.growth.HLRTGrowthController`
implements it for HLRT.  After every growth the optimizer is rebuilt through
``optimizer_factory`` (or an Adam with the old lr / weight decay).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Tuple

import torch
import torch.nn as nn


@dataclass
class GrowthEvent:
    step: int
    event_type: str
    description: str = ""
    old_param_count: int = 0
    new_param_count: int = 0
    metadata: Dict[str, Any] = field(default_factory=dict)


class GrowthController:
    def __init__(
        self,
        model: nn.Module,
        optimizer: torch.optim.Optimizer,
        schedule: Optional[List[Tuple[int, str, Dict[str, Any]]]] = None,
        patience: int = 500,
        min_delta: float = 0.001,
        optimizer_factory: Optional[Callable] = None,
    ) -> None:
        self.model = model
        self.optimizer = optimizer
        self.schedule = sorted(schedule or [], key=lambda e: e[0])
        self.patience = patience
        self.min_delta = min_delta
        self.optimizer_factory = optimizer_factory
        self._history: List[GrowthEvent] = []
        self._best_loss = float("inf")
        self._steps_without_improvement = 0
        self._completed_scheduled: set = set()

    def maybe_grow(self, step: int, current_loss: float) -> Optional[GrowthEvent]:
        for when, kind, kwargs in self.schedule:
            if when == step and when not in self._completed_scheduled:
                event = self._execute_growth(step, kind, kwargs)
                self._completed_scheduled.add(when)
                return event
        if current_loss < self._best_loss - self.min_delta:
            self._best_loss = current_loss
            self._steps_without_improvement = 0
        else:
            self._steps_without_improvement += 1
        if self._steps_without_improvement >= self.patience:
            event = self._execute_growth(step, "widen", {"factor": 1.5})
            self._steps_without_improvement = 0
            self._best_loss = current_loss
            return event
        return None

    @property
    def history(self) -> List[GrowthEvent]:
        return list(self._history)

    def _widen(self, model: nn.Module, factor: float = 2.0, **kwargs: Any) -> nn.Module:
        raise NotImplementedError("_widen() is architecture-specific; subclass GrowthController.")

    def _deepen(self, model: nn.Module, num_layers: int = 1, position: str = "end", **kwargs: Any) -> nn.Module:
        raise NotImplementedError("_deepen() is architecture-specific; subclass GrowthController.")

    def _dense_to_moe(self, model: nn.Module, num_experts: int = 4, top_k: int = 2, **kwargs: Any) -> nn.Module:
        raise NotImplementedError("_dense_to_moe() is architecture-specific; subclass GrowthController.")

    def _execute_growth(self, step: int, event_type: str, kwargs: Dict[str, Any]) -> GrowthEvent:
        ops = {"widen": self._widen, "deepen": self._deepen, "dense_to_moe": self._dense_to_moe}
        if event_type not in ops:
            raise ValueError(f"Unknown growth event type: '{event_type}'. Must be one of {list(ops)}.")
        before = sum(p.numel() for p in self.model.parameters())
        self.model = ops[event_type](self.model, **kwargs)
        after = sum(p.numel() for p in self.model.parameters())
        self.optimizer = self._migrate_optimizer()
        event = GrowthEvent(
            step=step,
            event_type=event_type,
            description=f"{event_type} at step {step} with {kwargs}",
            old_param_count=before,
            new_param_count=after,
            metadata=dict(kwargs),
        )
        self._history.append(event)
        return event

    def _migrate_optimizer(self) -> torch.optim.Optimizer:
        if self.optimizer_factory is not None:
            return self.optimizer_factory(self.model.parameters())
        defaults = dict(self.optimizer.defaults)
        return torch.optim.Adam(self.model.parameters(), lr=defaults.get("lr", 1e-4), weight_decay=defaults.get("weight_decay", 0.0))
