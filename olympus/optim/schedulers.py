"""Warmup-Stable-Decay learning-rate schedule (``olympus/optim/schedulers.py:10-147``).

``lr(step)``:
  * ``step < warmup_steps``:     ``base_lr * step / warmup_steps``
  * ``step < decay_start``:      ``base_lr``
  * otherwise:                   cosine from ``base_lr`` down to ``min_lr`` over
                                 ``total_steps - decay_start`` steps.
After :meth:`notify_growth`, the value is further multiplied by a linear
re-warmup over ``post_growth_warmup_steps`` steps.

Like the reference, :meth:`step` writes ``param_group["lr"]``.  The reference's
:class:`MuonAdamWHybrid` reads ``lr_muon``/``lr_adamw`` instead, so the schedule
never reaches it there.  ``drive_hybrid_lrs=True`` (off by default, to keep
the reference behaviour) also scales each group's ``lr_muon`` and
``lr_adamw`` by ``lr / base_lr`` relative to their values at construction.
"""

from __future__ import annotations

import math
from typing import Optional


class WSDScheduler:
    def __init__(
        self,
        optimizer,
        base_lr: float = 3e-4,
        min_lr: float = 1e-5,
        warmup_steps: int = 2000,
        total_steps: int = 100_000,
        decay_start: Optional[int] = None,
        decay_steps: Optional[int] = None,
        post_growth_warmup_steps: int = 500,
        drive_hybrid_lrs: bool = False,
    ) -> None:
        self.optimizer = optimizer
        self.base_lr = base_lr
        self.min_lr = min_lr
        self.warmup_steps = warmup_steps
        self.total_steps = total_steps
        self.post_growth_warmup_steps = post_growth_warmup_steps
        if decay_start is not None:
            self.decay_start = decay_start
        elif decay_steps is not None:
            self.decay_start = total_steps - decay_steps
        else:
            self.decay_start = int(total_steps * 0.8)
        self.drive_hybrid_lrs = drive_hybrid_lrs
        self._hybrid_base = [
            {k: g[k] for k in ("lr_muon", "lr_adamw") if k in g} for g in getattr(optimizer, "param_groups", [])
        ]
        self._step_count = 0
        self._growth_step: Optional[int] = None
        self._last_lr = 0.0

    def get_lr(self, step: Optional[int] = None) -> float:
        s = self._step_count if step is None else step
        if s < self.warmup_steps:
            lr = self.base_lr * s / max(self.warmup_steps, 1)
        elif s < self.decay_start:
            lr = self.base_lr
        else:
            span = max(self.total_steps - self.decay_start, 1)
            t = min((s - self.decay_start) / span, 1.0)
            lr = self.min_lr + 0.5 * (self.base_lr - self.min_lr) * (1.0 + math.cos(math.pi * t))
        if self._growth_step is not None:
            since = s - self._growth_step
            if 0 <= since < self.post_growth_warmup_steps:
                lr *= since / max(self.post_growth_warmup_steps, 1)
        return lr

    def step(self) -> None:
        lr = self.get_lr(self._step_count)
        self._last_lr = lr
        ratio = lr / self.base_lr if self.base_lr else 0.0
        for i, group in enumerate(self.optimizer.param_groups):
            group["lr"] = lr
            if self.drive_hybrid_lrs and i < len(self._hybrid_base):
                for key, base in self._hybrid_base[i].items():
                    group[key] = base * ratio
        self._step_count += 1

    def notify_growth(self, step: Optional[int] = None) -> None:
        self._growth_step = self._step_count if step is None else step

    @property
    def last_lr(self) -> float:
        return self._last_lr

    def state_dict(self) -> dict:
        return {
            "step_count": self._step_count,
            "growth_step": self._growth_step,
            "last_lr": self._last_lr,
            "base_lr": self.base_lr,
            "min_lr": self.min_lr,
            "warmup_steps": self.warmup_steps,
            "total_steps": self.total_steps,
            "decay_start": self.decay_start,
            "post_growth_warmup_steps": self.post_growth_warmup_steps,
        }

    def load_state_dict(self, state: dict) -> None:
        self._step_count = state["step_count"]
        self._growth_step = state.get("growth_step")
        self._last_lr = state.get("last_lr", 0.0)
        for key in ("base_lr", "min_lr", "warmup_steps", "total_steps", "decay_start", "post_growth_warmup_steps"):
            if key in state:
                setattr(self, key, state[key])
