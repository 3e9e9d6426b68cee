"""Phase 1: next-token-prediction bootstrap training
(``genesis/training/train_phase1_bootstrap.py:43-260``).

:func:`ntp_objective` is shifted cross-entropy plus the model's auxiliary
loss; on CUDA it is one fused kernel pass over the unshifted logits
(``llm_research_b200.ops.shifted_cross_entropy``).

:class:`BootstrapTrainer` wires HLRT, the optimizer and the scheduler into a
:class:`TrainingOrchestrator` (phase ``bootstrap``).  Config keys:
``gradient_accumulation_steps`` (4), ``max_grad_norm`` (1.0),
``log_interval`` (100), ``save_interval`` (5000), ``checkpoint_dir``,
``device`` (``"cuda"``), and two additions: ``precision`` (``"fp32"`` as in
the reference, or ``"bf16"`` for bf16 compute with fp32 master weights via
the flat-shard engine) and ``sync_metrics`` (True: losses are returned as
floats every micro-step; False: they stay on the device).
"""

from __future__ import annotations

import logging
import math
import os
import time
from typing import Any, Dict

import torch
import torch.nn as nn
from torch.utils.data import DataLoader

from genesis.model.hlrt import HLRT
from llm_research_b200.ops.loss import shifted_cross_entropy
from olympus.core.training_context import TrainingContext
from olympus.core.training_orchestrator import ModelConfig, ObjectiveConfig, TrainingOrchestrator
from olympus.data.tokenizer import TokenizerWrapper

logger = logging.getLogger(__name__)


def ntp_objective(models: Dict[str, nn.Module], ctx: TrainingContext, batch: Any) -> torch.Tensor:
    model = models["hlrt"]
    device = getattr(model, "device", None) or next(model.parameters()).device
    input_ids = batch["input_ids"]
    if input_ids.device != device:
        input_ids = input_ids.to(device, non_blocking=True)
    if batch.get("fused_lm_loss", False):  # extension: chunked head + CE, no full logits
        targets = torch.cat([input_ids[:, 1:], input_ids.new_full((input_ids.shape[0], 1), -100)], dim=1)
        out = model(input_ids, labels=targets)
        loss = out["lm_loss"]
    else:
        out = model(input_ids)
        loss = shifted_cross_entropy(out["logits"], input_ids, ignore_index=-100)
    aux = out.get("aux_loss", 0.0)
    if isinstance(aux, torch.Tensor):
        loss = loss + aux.to(loss.dtype)
    elif isinstance(aux, (int, float)) and aux > 0:
        loss = loss + aux
    return loss


def _to_float(v: Any) -> float:
    return float(v) if not isinstance(v, float) else v


class BootstrapTrainer:
    def __init__(self, model: HLRT, optimizer, scheduler, tokenizer: TokenizerWrapper, config: dict) -> None:
        self.config = config
        self.device = torch.device(config.get("device", "cuda"))
        self.model = model.to(self.device)
        self.optimizer = optimizer
        self.scheduler = scheduler
        self.tokenizer = tokenizer
        accum = config.get("gradient_accumulation_steps", 4)
        sync = config.get("sync_metrics", True)
        if config.get("precision", "fp32") in ("bf16", "fp16"):
            from olympus.distributed.distributed_orchestrator import DistributedTrainingOrchestrator
            from olympus.distributed.fsdp_wrapper import FSDPConfig

            self.orchestrator: TrainingOrchestrator = DistributedTrainingOrchestrator(
                fsdp_config=FSDPConfig(mixed_precision=config["precision"],
                                       activation_checkpointing=config.get("activation_checkpointing", False)),
                gradient_accumulation_steps=accum, device=self.device, sync_metrics=sync,
            )
        else:
            self.orchestrator = TrainingOrchestrator(gradient_accumulation_steps=accum, device=self.device, sync_metrics=sync)
        self.orchestrator.add_model(ModelConfig(
            name="hlrt", model=self.model, optimizer=self.optimizer, scheduler=self.scheduler,
            max_grad_norm=config.get("max_grad_norm", 1.0), enabled_phases=["bootstrap"],
        ))
        self.orchestrator.add_objective(ObjectiveConfig(
            name="ntp", compute_fn=ntp_objective, weight=1.0, enabled_phases=["bootstrap"],
        ))
        self.orchestrator.set_phase("bootstrap")
        cfg = self.orchestrator._models["hlrt"]
        self.model, self.optimizer, self.scheduler = cfg.model, cfg.optimizer, cfg.scheduler
        self._tokens_seen = 0
        logger.info("HLRT model: %.2fM parameters", sum(p.numel() for p in model.parameters()) / 1e6)

    def train_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, Any]:
        t0 = time.time()
        losses = self.orchestrator.step(batch)
        total = losses.get("total", losses.get("ntp", 0.0))
        n = batch["input_ids"].numel()
        self._tokens_seen += n
        out: Dict[str, Any] = {"loss": total, "lr": getattr(self.scheduler, "last_lr", 0.0)}
        if isinstance(total, torch.Tensor):
            out["perplexity"] = torch.where(total < 20, total.exp().clamp(max=1e6), torch.full_like(total, 1e6))
        else:
            out["perplexity"] = min(math.exp(total), 1e6) if total < 20 else 1e6
        out["tokens_per_sec"] = n / max(time.time() - t0, 1e-6)
        return out

    def train_epoch(self, dataloader: DataLoader) -> Dict[str, float]:
        log_every = self.config.get("log_interval", 100)
        save_every = self.config.get("save_interval", 5000)
        ckpt_dir = self.config.get("checkpoint_dir", "checkpoints/phase1")
        total_loss, total_tps, steps = 0.0, 0.0, 0
        start = time.time()
        for batch in dataloader:
            m = self.train_step(batch)
            loss = _to_float(m["loss"])
            total_loss += loss
            total_tps += m["tokens_per_sec"]
            steps += 1
            gs = self.orchestrator.global_step
            if steps % log_every == 0:
                logger.info("Step %d | loss=%.4f | lr=%.2e | %.0f tok/s", gs, loss, m["lr"], m["tokens_per_sec"])
            if save_every > 0 and gs > 0 and gs % save_every == 0 and self.orchestrator._accumulation_step == 0:
                self.save_checkpoint(os.path.join(ckpt_dir, f"checkpoint_step{gs}.pt"))
        avg = total_loss / max(steps, 1)
        logger.info("Epoch complete | avg_loss=%.4f | %d steps in %.1fs", avg, steps, time.time() - start)
        return {
            "epoch_loss": avg,
            "epoch_perplexity": min(math.exp(avg), 1e6) if avg < 20 else 1e6,
            "avg_tokens_per_sec": total_tps / max(steps, 1),
            "total_steps": steps,
        }

    def save_checkpoint(self, path: str) -> None:
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        self.orchestrator.save_checkpoint(path)

    def load_checkpoint(self, path: str) -> None:
        self.orchestrator.load_checkpoint(path)
