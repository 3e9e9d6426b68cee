"""Progressive model growth (reference: ``olympus/core/growth_controller.py:17-210``).

A :class:`GrowthController` decides *when* a model grows and keeps the record;
the tensor surgery that decides *how* is a set of hooks a model family
overrides -- ``_widen``, ``_deepen`` and ``_dense_to_moe``, each taking the
model and returning the grown model.  The base class raises
``NotImplementedError`` from all three; :class:`genesis.model.growth.HLRTGrowthController`
implements them for HLRT with function-preserving surgery.

When growth fires:

* on a schedule: ``(step, kind, kwargs)`` entries; each fires once, the first
  time ``maybe_grow`` is called at exactly that step (several entries for one
  step fire on successive calls at that step);
* adaptively: a plateau of ``patience`` consecutive calls without the loss
  beating the best seen by more than ``min_delta`` triggers
  ``widen(factor=1.5)`` and restarts the plateau count from the current loss.

After a growth the optimizer is rebuilt over the new parameters: with
``optimizer_factory`` when given, otherwise as the same optimizer class with
the old optimizer's defaults; per-parameter state (momentum, moments) is
carried over for every parameter tensor that survived the surgery unchanged
in shape.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterable, List, Optional, Tuple

import torch
import torch.nn as nn

GROWTH_KINDS = ("widen", "deepen", "dense_to_moe")


@dataclass
class GrowthEvent:
    """One growth: when, what, and the parameter count before and after."""

    step: int
    event_type: str
    description: str = ""
    old_param_count: int = 0
    new_param_count: int = 0
    metadata: Dict[str, Any] = field(default_factory=dict)


class _Plateau:
    """Counts calls since the loss last improved on its best by more than ``delta``."""

    def __init__(self, patience: int, delta: float) -> None:
        self.patience, self.delta = patience, delta
        self.best = float("inf")
        self.stale = 0

    def update(self, loss: float) -> bool:
        """Record ``loss``; True when the plateau has lasted ``patience`` calls."""
        if loss < self.best - self.delta:
            self.best, self.stale = loss, 0
        else:
            self.stale += 1
        return self.stale >= self.patience

    def restart(self, loss: float) -> None:
        self.best, self.stale = loss, 0


def _param_count(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


class GrowthController:
    def __init__(
        self,
        model: nn.Module,
        optimizer: torch.optim.Optimizer,
        schedule: Optional[List[Tuple[int, str, Dict[str, Any]]]] = None,
        patience: int = 500,
        min_delta: float = 0.001,
        optimizer_factory: Optional[Callable[[Iterable[nn.Parameter]], torch.optim.Optimizer]] = None,
    ) -> None:
        self.model = model
        self.optimizer = optimizer
        self.optimizer_factory = optimizer_factory
        self.patience = patience
        self.min_delta = min_delta
        # step -> growths still to run at that step, in schedule order
        self._pending: Dict[int, List[Tuple[str, Dict[str, Any]]]] = {}
        for step, kind, kwargs in schedule or []:
            self._pending.setdefault(int(step), []).append((kind, dict(kwargs or {})))
        self.schedule = sorted(((s, k, kw) for s, lst in self._pending.items() for k, kw in lst), key=lambda e: e[0])
        self._plateau = _Plateau(patience, min_delta)
        self._events: List[GrowthEvent] = []

    # ----------------------------------------------------------- decisions
    def maybe_grow(self, step: int, current_loss: float) -> Optional[GrowthEvent]:
        """Called once per training step with the step's loss; returns the growth
        performed at this call, if any."""
        due = self._pending.get(step)
        if due:
            kind, kwargs = due.pop(0)
            if not due:
                del self._pending[step]
            return self._grow(step, kind, kwargs)
        if self._plateau.update(float(current_loss)):
            self._plateau.restart(float(current_loss))
            return self._grow(step, "widen", {"factor": 1.5})
        return None

    @property
    def history(self) -> List[GrowthEvent]:
        return list(self._events)

    # ------------------------------------------------------ surgery hooks
    def _widen(self, model: nn.Module, factor: float = 2.0, **kwargs: Any) -> nn.Module:
        raise NotImplementedError(f"{type(self).__name__} has no widen surgery for {type(model).__name__}")

    def _deepen(self, model: nn.Module, num_layers: int = 1, position: str = "end", **kwargs: Any) -> nn.Module:
        raise NotImplementedError(f"{type(self).__name__} has no deepen surgery for {type(model).__name__}")

    def _dense_to_moe(self, model: nn.Module, num_experts: int = 4, top_k: int = 2, **kwargs: Any) -> nn.Module:
        raise NotImplementedError(f"{type(self).__name__} has no dense-to-MoE surgery for {type(model).__name__}")

    # ------------------------------------------------------------ execution
    def _grow(self, step: int, kind: str, kwargs: Dict[str, Any]) -> GrowthEvent:
        if kind not in GROWTH_KINDS:
            raise ValueError(f"Unknown growth event type: '{kind}'. Must be one of {list(GROWTH_KINDS)}.")
        before = _param_count(self.model)
        old_params = list(self.model.parameters())
        self.model = getattr(self, "_" + kind)(self.model, **kwargs)
        self.optimizer = self._rebuild_optimizer(old_params)
        event = GrowthEvent(step=step, event_type=kind, description=f"{kind} at step {step} with {kwargs}",
                            old_param_count=before, new_param_count=_param_count(self.model), metadata=dict(kwargs))
        self._events.append(event)
        return event

    def _rebuild_optimizer(self, old_params: List[nn.Parameter]) -> torch.optim.Optimizer:
        params = list(self.model.parameters())
        if self.optimizer_factory is not None:
            new = self.optimizer_factory(params)
        else:
            import inspect

            cls = type(self.optimizer)
            accepted = inspect.signature(cls.__init__).parameters
            kw = {k: v for k, v in self.optimizer.defaults.items() if k in accepted}
            new = cls(params, **kw)
        old_state = self.optimizer.state
        survivors = {id(p) for p in old_params}
        for p in params:
            st = old_state.get(p)
            if not st or id(p) not in survivors:
                continue
            # state tensors shaped like the parameter must still match it
            if all(not torch.is_tensor(v) or v.dim() == 0 or v.shape == p.shape for v in st.values()):
                new.state[p] = st
        return new
