"""Multi-model, multi-objective training loop (``olympus/core/training_orchestrator.py``).

One :meth:`TrainingOrchestrator.step` call is one micro-step:

1. build a :class:`TrainingContext`;
2. put the models active in the current phase into train mode;
3. evaluate every active objective and sum them with their weights;
4. backward of ``total / gradient_accumulation_steps``;
5. on the accumulation boundary: clip, optimizer step, zero grads, scheduler
   step, advance ``global_step``;
6. clear the ``step`` scope of the memory bus.

Checkpoints use the reference layout (global_step, epoch, phase, prev_loss,
memory_bus, models, optimizers, schedulers).

``sync_metrics=False`` keeps the per-objective losses on the device (returned
as detached 0-d tensors) so a micro-step never waits for the GPU; the default
returns Python floats exactly like the reference.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional

import torch
import torch.nn as nn

from olympus.core.memory_bus import MemoryBus
from olympus.core.stateful_module import StatefulModule
from olympus.core.training_context import TrainingContext

logger = logging.getLogger(__name__)


@dataclass
class ModelConfig:
    name: str
    model: nn.Module
    optimizer: torch.optim.Optimizer
    scheduler: Optional[Any] = None
    max_grad_norm: float = 1.0
    enabled_phases: Optional[List[str]] = None

    def is_active(self, phase: str) -> bool:
        return self.enabled_phases is None or phase in self.enabled_phases


@dataclass
class ObjectiveConfig:
    """``compute_fn(models: Dict[str, nn.Module], ctx, batch) -> scalar loss``."""

    name: str
    compute_fn: Callable[..., torch.Tensor]
    weight: float = 1.0
    enabled_phases: Optional[List[str]] = None

    def is_active(self, phase: str) -> bool:
        return self.enabled_phases is None or phase in self.enabled_phases


def rng_state() -> Dict[str, Any]:
    """Python, NumPy, torch CPU and (when present) this process's CUDA generator
    states: an extension of the reference's checkpoint, which saves none, so a
    resumed run draws the same dropout masks, jitter and samples as an
    uninterrupted one.  Readers of the reference ignore the extra key.  Only
    tensors, numbers and strings, so ``weights_only`` loaders accept it."""
    import random

    import numpy as np

    kind, keys, pos, has_gauss, gauss = np.random.get_state()
    out: Dict[str, Any] = {"python": random.getstate(),
                           "numpy": (kind, torch.from_numpy(keys.astype(np.int64)), int(pos), int(has_gauss),
                                     float(gauss)),
                           "torch": torch.get_rng_state()}
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        out["cuda"] = torch.cuda.get_rng_state()
    return out


def set_rng_state(state: Dict[str, Any]) -> None:
    import random

    import numpy as np

    random.setstate(state["python"])
    kind, keys, pos, has_gauss, gauss = state["numpy"]
    np.random.set_state((kind, np.asarray(keys, dtype=np.int64).astype(np.uint32), pos, has_gauss, gauss))
    torch.set_rng_state(state["torch"].cpu())
    if "cuda" in state and torch.cuda.is_available():
        torch.cuda.set_rng_state(state["cuda"].cpu())


def model_state_for_checkpoint(model: nn.Module) -> Dict[str, Any]:
    if isinstance(model, StatefulModule):
        return model.state_dict_with_state()
    return model.state_dict()


def load_model_state(model: nn.Module, state: Dict[str, Any], strict: bool = True) -> None:
    state = dict(state)
    if isinstance(model, StatefulModule):
        model.load_state_dict_with_state(state, strict=strict)
    else:
        for k in [k for k in state if k.startswith("_olympus_")]:
            state.pop(k)
        model.load_state_dict(state, strict=strict)


class TrainingOrchestrator:
    def __init__(
        self,
        memory_bus: Optional[MemoryBus] = None,
        gradient_accumulation_steps: int = 1,
        device: Optional[torch.device] = None,
        sync_metrics: bool = True,
    ) -> None:
        self.memory_bus = memory_bus or MemoryBus()
        self.gradient_accumulation_steps = int(gradient_accumulation_steps)
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.sync_metrics = sync_metrics
        self._models: Dict[str, ModelConfig] = {}
        self._objectives: Dict[str, ObjectiveConfig] = {}
        self._phase = "bootstrap"
        self._global_step = 0
        self._epoch = 0
        # further top-level checkpoint entries set by the trainer (its data position, say)
        self.extra_state: Dict[str, Any] = {}
        self._prev_loss: Any = float("inf")
        self._accumulation_step = 0

    # ------------------------------------------------------------ registration
    def add_model(self, config: ModelConfig) -> None:
        if config.name in self._models:
            raise ValueError(f"Model '{config.name}' is already registered.")
        self._models[config.name] = config
        logger.info("Registered model '%s' (%d params)", config.name, sum(p.numel() for p in config.model.parameters()))

    def add_objective(self, config: ObjectiveConfig) -> None:
        if config.name in self._objectives:
            raise ValueError(f"Objective '{config.name}' is already registered.")
        self._objectives[config.name] = config

    def set_phase(self, phase: str) -> None:
        logger.info("Phase transition: %s -> %s", self._phase, phase)
        self._phase = phase

    def set_epoch(self, epoch: int) -> None:
        self._epoch = epoch

    @property
    def global_step(self) -> int:
        return self._global_step

    @property
    def phase(self) -> str:
        return self._phase

    @property
    def prev_loss(self) -> float:
        if isinstance(self._prev_loss, torch.Tensor):
            self._prev_loss = float(self._prev_loss)
        return self._prev_loss

    # ---------------------------------------------------------------- hooks
    def _active_models(self) -> Dict[str, ModelConfig]:
        return {n: c for n, c in self._models.items() if c.is_active(self._phase)}

    def _active_objectives(self) -> Dict[str, ObjectiveConfig]:
        return {n: c for n, c in self._objectives.items() if c.is_active(self._phase)}

    def _make_context(self) -> TrainingContext:
        return TrainingContext(
            global_step=self._global_step,
            epoch=self._epoch,
            phase=self._phase,
            prev_loss=self.prev_loss if self.sync_metrics else float("nan"),
            is_training=True,
            gradient_accumulation_steps=self.gradient_accumulation_steps,
            current_accumulation_step=self._accumulation_step,
            memory_bus=self.memory_bus,
        )

    def _is_boundary_next(self) -> bool:
        return self._accumulation_step + 1 >= self.gradient_accumulation_steps

    def _backward(self, loss: torch.Tensor, active: Dict[str, ModelConfig]) -> None:
        loss.backward()

    def _clip(self, cfg: ModelConfig) -> None:
        if cfg.max_grad_norm > 0:
            clip = getattr(cfg.model, "clip_grad_norm_", None)
            if callable(clip):
                clip(cfg.max_grad_norm)
            else:
                nn.utils.clip_grad_norm_(cfg.model.parameters(), cfg.max_grad_norm)

    def _optimizer_step(self, cfg: ModelConfig) -> None:
        cfg.optimizer.step()
        cfg.optimizer.zero_grad(set_to_none=True)
        if cfg.scheduler is not None:
            cfg.scheduler.step()

    def _value(self, t: torch.Tensor) -> Any:
        return float(t.detach()) if self.sync_metrics else t.detach()

    # ----------------------------------------------------------------- step
    def step(self, batch: Any) -> Dict[str, Any]:
        ctx = self._make_context()
        active = self._active_models()
        objectives = self._active_objectives()
        for cfg in active.values():
            cfg.model.train()
        models = {n: c.model for n, c in active.items()}

        losses: Dict[str, Any] = {}
        total: Optional[torch.Tensor] = None
        for name, obj in objectives.items():
            loss = obj.compute_fn(models, ctx, batch)
            losses[name] = self._value(loss)
            term = obj.weight * loss
            total = term if total is None else total + term
        if total is None:
            total = torch.zeros((), device=self.device, requires_grad=True)

        self._backward(total / self.gradient_accumulation_steps, active)
        losses["total"] = self._value(total)

        self._accumulation_step += 1
        if self._accumulation_step >= self.gradient_accumulation_steps:
            self._accumulation_step = 0
            for cfg in active.values():
                self._clip(cfg)
                self._optimizer_step(cfg)
            self._global_step += 1
            self._prev_loss = losses["total"]
        self.memory_bus.step()
        return losses

    # ----------------------------------------------------------- checkpoints
    def _checkpoint_dict(self) -> Dict[str, Any]:
        return {
            "global_step": self._global_step,
            "epoch": self._epoch,
            "phase": self._phase,
            "prev_loss": self.prev_loss,
            "memory_bus": self.memory_bus.state_dict(),
            "models": {},
            "optimizers": {},
            "schedulers": {},
            "rng_state": rng_state(),
            **self.extra_state,
        }

    def save_checkpoint(self, path: str) -> None:
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        ckpt = self._checkpoint_dict()
        for name, cfg in self._models.items():
            ckpt["models"][name] = model_state_for_checkpoint(cfg.model)
            ckpt["optimizers"][name] = cfg.optimizer.state_dict()
            if cfg.scheduler is not None and hasattr(cfg.scheduler, "state_dict"):
                ckpt["schedulers"][name] = cfg.scheduler.state_dict()
        torch.save(ckpt, path)
        logger.info("Checkpoint saved to %s (step %d)", path, self._global_step)

    def _restore_header(self, ckpt: Dict[str, Any]) -> None:
        self._global_step = ckpt["global_step"]
        self._epoch = ckpt["epoch"]
        self._phase = ckpt["phase"]
        self._prev_loss = ckpt["prev_loss"]
        self.memory_bus.load_state_dict(ckpt["memory_bus"])
        self._restore_rng(ckpt)

    def _restore_rng(self, ckpt: Dict[str, Any]) -> None:
        if "rng_state" in ckpt:  # absent in the reference's checkpoints
            set_rng_state(ckpt["rng_state"])

    def load_checkpoint(self, path: str, strict: bool = True) -> Dict[str, Any]:
        ckpt = torch.load(path, map_location=self.device, weights_only=False)
        self._restore_header(ckpt)
        for name, cfg in self._models.items():
            if name in ckpt["models"]:
                load_model_state(cfg.model, ckpt["models"][name], strict=strict)
            if name in ckpt["optimizers"]:
                cfg.optimizer.load_state_dict(ckpt["optimizers"][name])
            if cfg.scheduler is not None and name in ckpt.get("schedulers", {}):
                cfg.scheduler.load_state_dict(ckpt["schedulers"][name])
        logger.info("Checkpoint loaded from %s (step %d)", path, self._global_step)
        return ckpt
