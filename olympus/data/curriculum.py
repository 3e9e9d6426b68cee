"""Multi-phase training curriculum (``olympus/data/curriculum.py:16-318``).

Phases run in order bootstrap -> rl_pretrain -> flywheel -> vision.  Each has
a base data mix, optional time-varying ``mix_schedule`` (piecewise-linear
interpolation between ``(phase_step, mix)`` points, renormalised), and a
transition rule: after ``min_steps`` within the phase, move on once
``transition_metric`` is ``below``/``above`` ``transition_threshold``; always
move on after ``max_steps``.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

logger = logging.getLogger(__name__)


@dataclass
class PhaseConfig:
    name: str
    base_mix: Dict[str, float] = field(default_factory=lambda: {"web": 1.0})
    min_steps: int = 0
    max_steps: int = 100_000
    transition_metric: str = "loss"
    transition_threshold: float = 2.0
    transition_direction: str = "below"
    mix_schedule: List[Tuple[int, Dict[str, float]]] = field(default_factory=list)


DEFAULT_PHASES: Dict[str, PhaseConfig] = {
    "bootstrap": PhaseConfig(
        name="bootstrap", base_mix={"web": 0.7, "books": 0.2, "code": 0.1}, min_steps=5000, max_steps=200_000,
        transition_metric="loss", transition_threshold=2.5, transition_direction="below",
        mix_schedule=[(0, {"web": 0.7, "books": 0.2, "code": 0.1}),
                      (50_000, {"web": 0.6, "books": 0.25, "code": 0.15}),
                      (100_000, {"web": 0.5, "books": 0.3, "code": 0.2})],
    ),
    "rl_pretrain": PhaseConfig(
        name="rl_pretrain", base_mix={"web": 0.4, "reasoning": 0.4, "code": 0.2}, min_steps=2000, max_steps=100_000,
        transition_metric="avg_reward", transition_threshold=0.5, transition_direction="above",
    ),
    "flywheel": PhaseConfig(
        name="flywheel", base_mix={"web": 0.3, "reasoning_traces": 0.4, "code": 0.15, "books": 0.15},
        min_steps=5000, max_steps=500_000, transition_metric="loss", transition_threshold=1.5,
        transition_direction="below",
    ),
    "vision": PhaseConfig(
        name="vision", base_mix={"web": 0.3, "image_text": 0.4, "code": 0.1, "reasoning_traces": 0.2},
        min_steps=5000, max_steps=200_000, transition_metric="loss", transition_threshold=1.8,
        transition_direction="below",
    ),
}
DEFAULT_PHASE_ORDER: List[str] = ["bootstrap", "rl_pretrain", "flywheel", "vision"]


def _interpolate(schedule: List[Tuple[int, Dict[str, float]]], t: int) -> Dict[str, float]:
    pts = sorted(schedule, key=lambda p: p[0])
    if t <= pts[0][0]:
        return dict(pts[0][1])
    if t >= pts[-1][0]:
        return dict(pts[-1][1])
    for (s0, m0), (s1, m1) in zip(pts, pts[1:]):
        if s0 <= t < s1:
            a = (t - s0) / max(s1 - s0, 1)
            mix = {k: m0.get(k, 0.0) + a * (m1.get(k, 0.0) - m0.get(k, 0.0)) for k in set(m0) | set(m1)}
            tot = sum(mix.values())
            return {k: v / tot for k, v in mix.items()} if tot > 0 else mix
    return dict(pts[-1][1])


class Curriculum:
    def __init__(self, phases: Optional[Dict[str, PhaseConfig]] = None, phase_order: Optional[List[str]] = None) -> None:
        self.phases = phases or dict(DEFAULT_PHASES)
        self.phase_order = phase_order or list(DEFAULT_PHASE_ORDER)
        self._current_phase_idx = 0
        self._phase_start_step = 0
        self._transition_history: List[Dict[str, Any]] = []

    @property
    def current_phase(self) -> str:
        return self.phase_order[min(self._current_phase_idx, len(self.phase_order) - 1)]

    @property
    def current_phase_config(self) -> PhaseConfig:
        return self.phases[self.current_phase]

    @property
    def is_final_phase(self) -> bool:
        return self._current_phase_idx >= len(self.phase_order) - 1

    def get_mix_ratios(self, phase: Optional[str] = None, step: int = 0) -> Dict[str, float]:
        phase = phase or self.current_phase
        cfg = self.phases.get(phase)
        if cfg is None:
            logger.warning("Unknown phase %r, returning uniform mix", phase)
            return {"web": 1.0}
        if not cfg.mix_schedule:
            return dict(cfg.base_mix)
        return _interpolate(cfg.mix_schedule, step - self._phase_start_step)

    def should_transition(self, metrics: Dict[str, float], step: int) -> bool:
        if self.is_final_phase:
            return False
        cfg = self.current_phase_config
        in_phase = step - self._phase_start_step
        if in_phase >= cfg.max_steps:
            return True
        if in_phase < cfg.min_steps:
            return False
        val = metrics.get(cfg.transition_metric)
        if val is None:
            return False
        return val < cfg.transition_threshold if cfg.transition_direction == "below" else val > cfg.transition_threshold

    def transition(self, step: int, metrics: Optional[Dict[str, float]] = None) -> str:
        old = self.current_phase
        if not self.is_final_phase:
            self._current_phase_idx += 1
        self._transition_history.append({"from": old, "to": self.current_phase, "step": step,
                                         "metrics": dict(metrics or {})})
        self._phase_start_step = step
        logger.info("Curriculum: %s -> %s at step %d", old, self.current_phase, step)
        return self.current_phase

    def set_phase(self, phase: str, step: int = 0) -> None:
        if phase not in self.phase_order:
            raise ValueError(f"Unknown phase {phase!r}; known: {self.phase_order}")
        self._current_phase_idx = self.phase_order.index(phase)
        self._phase_start_step = step

    @property
    def transition_history(self) -> List[Dict[str, Any]]:
        return list(self._transition_history)

    def state_dict(self) -> Dict[str, Any]:
        return {"current_phase_idx": self._current_phase_idx, "phase_start_step": self._phase_start_step,
                "transition_history": self._transition_history}

    def load_state_dict(self, state: Dict[str, Any]) -> None:
        self._current_phase_idx = state["current_phase_idx"]
        self._phase_start_step = state["phase_start_step"]
        self._transition_history = state.get("transition_history", [])
