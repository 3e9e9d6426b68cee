"""Sharded-data-parallel training orchestrator (``olympus/distributed/distributed_orchestrator.py:39-325``).

Drop-in replacement for :class:`TrainingOrchestrator`:

* ``add_model`` moves the model to the device, wraps it with
  :func:`~olympus.distributed.fsdp_wrapper.wrap_model_fsdp` and builds the
  sharded optimizer from the class and defaults of the optimizer passed in
  (distributed Muon for ``MuonAdamWHybrid``/``Muon``).  The scheduler is
  re-pointed at the new optimizer -- the reference rebuilds the optimizer
  and leaves its scheduler driving the discarded one
  (``distributed_orchestrator.py:95-102``).
* non-boundary micro-steps skip the gradient reduce-scatter (``no_sync``);
* clipping uses the global norm over all shards (one all-reduce);
* checkpoints gather the full state to rank 0 in the reference layout
  (plus ``world_size``), so they load into the single-process
  :class:`TrainingOrchestrator` and vice versa.

The wrapping is also used with ``world_size == 1`` whenever an
``fsdp_config`` is given: it provides bf16 compute with fp32 master weights
and fp32 gradient accumulation.
"""

from __future__ import annotations

import logging
import os
from typing import Any, Dict, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from olympus.core.memory_bus import MemoryBus
from olympus.core.stateful_module import StatefulModule
from olympus.core.training_orchestrator import (ModelConfig, ObjectiveConfig, TrainingOrchestrator, load_model_state,
                                               rng_state, set_rng_state)
from olympus.distributed.fsdp_wrapper import FSDPConfig, wrap_model_fsdp

logger = logging.getLogger(__name__)


def _is_engine(model: nn.Module) -> bool:
    from llm_research_b200.parallel.fsdp import FlatShardEngine

    return isinstance(model, FlatShardEngine)


def _engine_extra_state(engine) -> Dict[str, Any]:
    """Persistent buffers and Olympus state extras of an engine-wrapped model (host copies)."""
    out: Dict[str, Any] = {}
    inner = engine.module
    for bname, buf in inner.named_buffers():
        if not any(bname.endswith(x) for x in ("inv_freq", "cos_cached", "sin_cached")) and "_state_buf_" not in bname:
            out[bname] = buf.detach().cpu().clone()
    if isinstance(inner, StatefulModule):
        out.update(inner.olympus_extras())
    return out


class DistributedTrainingOrchestrator(TrainingOrchestrator):
    def __init__(
        self,
        fsdp_config: Optional[FSDPConfig] = None,
        local_rank: int = 0,
        world_size: int = 1,
        memory_bus: Optional[MemoryBus] = None,
        gradient_accumulation_steps: int = 1,
        device: Optional[torch.device] = None,
        sync_metrics: bool = True,
    ) -> None:
        if device is None:
            device = torch.device(f"cuda:{local_rank}") if torch.cuda.is_available() else torch.device("cpu")
        super().__init__(memory_bus=memory_bus, gradient_accumulation_steps=gradient_accumulation_steps,
                         device=device, sync_metrics=sync_metrics)
        self.fsdp_config = fsdp_config
        self.local_rank = local_rank
        self.world_size = world_size
        self._fsdp_enabled = fsdp_config is not None

    @property
    def is_main_rank(self) -> bool:
        return (dist.get_rank() if dist.is_initialized() else self.local_rank) == 0

    def add_model(self, config: ModelConfig) -> None:
        if self._fsdp_enabled:
            config.model = config.model.to(self.device)
            old = config.optimizer
            engine = wrap_model_fsdp(config.model, self.fsdp_config,
                                     device_id=self.device.index if self.device.type == "cuda" else None)
            config.model = engine
            config.optimizer = engine.make_optimizer(type(old), {k: v for k, v in old.defaults.items() if k != "params"})
            if config.scheduler is not None and hasattr(config.scheduler, "optimizer"):
                config.scheduler.optimizer = config.optimizer
                if hasattr(config.scheduler, "_hybrid_base"):
                    config.scheduler._hybrid_base = [
                        {k: g[k] for k in ("lr_muon", "lr_adamw") if k in g} for g in config.optimizer.param_groups
                    ]
        super().add_model(config)

    def _backward(self, loss: torch.Tensor, active: Dict[str, ModelConfig]) -> None:
        boundary = self._is_boundary_next()
        for cfg in active.values():
            if _is_engine(cfg.model):
                cfg.model.set_sync(boundary)
        loss.backward()

    def step(self, batch: Any) -> Dict[str, Any]:
        return super().step(batch)

    # ----------------------------------------------------------- checkpoints
    def save_checkpoint(self, path: str) -> None:
        if self.is_main_rank:
            os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        ckpt = self._checkpoint_dict()
        ckpt["world_size"] = self.world_size
        if dist.is_initialized():  # every rank's generators, restored rank by rank
            states: list = [None] * dist.get_world_size()
            dist.all_gather_object(states, ckpt["rng_state"])
            ckpt["rng_state"] = states
        for name, cfg in self._models.items():
            if _is_engine(cfg.model):
                state: Dict[str, Any] = dict(cfg.model.full_state_dict())
                state.update(_engine_extra_state(cfg.model))
                ckpt["models"][name] = state
            elif isinstance(cfg.model, StatefulModule):
                ckpt["models"][name] = cfg.model.state_dict_with_state()
            else:
                ckpt["models"][name] = cfg.model.state_dict()
            ckpt["optimizers"][name] = cfg.optimizer.state_dict()
            if cfg.scheduler is not None and hasattr(cfg.scheduler, "state_dict"):
                ckpt["schedulers"][name] = cfg.scheduler.state_dict()
        if self.is_main_rank:
            torch.save(ckpt, path)
            logger.info("Checkpoint saved to %s (step %d)", path, self._global_step)
        if dist.is_initialized():
            dist.barrier()

    def _restore_rng(self, ckpt: Dict[str, Any]) -> None:
        state = ckpt.get("rng_state")
        world = dist.get_world_size() if dist.is_initialized() else 1
        if isinstance(state, list):  # one entry per rank of the saving job
            if len(state) == world:
                set_rng_state(state[dist.get_rank() if dist.is_initialized() else 0])
        elif state is not None and world == 1:
            set_rng_state(state)

    def save_sharded_checkpoint(self, directory: str, asynchronous: bool = True) -> None:
        """Every rank writes its own parameter and optimizer shards (``{directory}/{model}/rank*.pt``)
        from a background thread; rank 0 writes ``header.pt`` (step, phase, memory bus, schedulers,
        models not wrapped by the engine). ``llm_research_b200.parallel.checkpoint.consolidate_checkpoint``
        turns the directory into the single-file layout that ``load_checkpoint`` reads."""
        from llm_research_b200.parallel import checkpoint as ck

        ck.wait()  # one checkpoint in flight at a time
        head = self._checkpoint_dict()
        head["world_size"] = dist.get_world_size() if dist.is_initialized() else self.world_size
        head["sharded"] = []
        for name, cfg in self._models.items():
            if _is_engine(cfg.model):
                ck.save_sharded(cfg.model, cfg.optimizer, os.path.join(directory, name),
                                header={"buffers": _engine_extra_state(cfg.model)}, asynchronous=asynchronous,
                                rank_extra={"rng_state": rng_state()})
                head["sharded"].append(name)
            else:
                head["models"][name] = (cfg.model.state_dict_with_state() if isinstance(cfg.model, StatefulModule)
                                        else cfg.model.state_dict())
                head["optimizers"][name] = cfg.optimizer.state_dict()
            if cfg.scheduler is not None and hasattr(cfg.scheduler, "state_dict"):
                head["schedulers"][name] = cfg.scheduler.state_dict()
        if self.is_main_rank:
            os.makedirs(directory, exist_ok=True)
            torch.save(head, os.path.join(directory, "header.pt"))
        if not asynchronous and dist.is_initialized():
            dist.barrier()

    def load_sharded_checkpoint(self, directory: str) -> Dict[str, Any]:
        from llm_research_b200.parallel import checkpoint as ck

        ck.wait()
        if dist.is_initialized():
            dist.barrier()  # every rank's writer has finished
        head = torch.load(os.path.join(directory, "header.pt"), map_location="cpu", weights_only=False)
        self._restore_header(head)
        for name, cfg in self._models.items():
            if name in head["sharded"]:
                sub = ck.load_sharded(cfg.model, cfg.optimizer, os.path.join(directory, name))
                if "rng_state" in sub:  # this rank's generators (same world size only)
                    set_rng_state(sub["rng_state"])
                extras = {k: v for k, v in sub.get("buffers", {}).items() if k.startswith("_olympus_")}
                inner = cfg.model.module
                if isinstance(inner, StatefulModule) and extras:
                    inner.restore_olympus_extras(extras)
            elif name in head["models"]:
                load_model_state(cfg.model, head["models"][name], strict=True)
                cfg.optimizer.load_state_dict(head["optimizers"][name])
            if cfg.scheduler is not None and name in head.get("schedulers", {}):
                cfg.scheduler.load_state_dict(head["schedulers"][name])
        return head

    def load_checkpoint(self, path: str, strict: bool = True) -> Dict[str, Any]:
        ckpt = torch.load(path, map_location="cpu", weights_only=False)
        self._restore_header(ckpt)
        for name, cfg in self._models.items():
            if name in ckpt["models"]:
                state = dict(ckpt["models"][name])
                if _is_engine(cfg.model):
                    extras = {k: state.pop(k) for k in list(state) if k.startswith("_olympus_")}
                    inner = cfg.model.module
                    if isinstance(inner, StatefulModule) and extras:
                        inner.restore_olympus_extras(extras)
                    pnames = {i.name for i in cfg.model.params}
                    if strict:
                        missing = pnames - set(state)
                        if missing:
                            raise KeyError(f"missing parameters in checkpoint: {sorted(missing)[:5]}")
                    cfg.model.load_full_state_dict({k: v for k, v in state.items() if k in pnames})
                else:
                    load_model_state(cfg.model, state, strict=strict)
            if name in ckpt["optimizers"]:
                cfg.optimizer.load_state_dict(ckpt["optimizers"][name])
            if cfg.scheduler is not None and name in ckpt.get("schedulers", {}):
                cfg.scheduler.load_state_dict(ckpt["schedulers"][name])
        return ckpt
