"""Phase 2: next-token prediction mixed with GRPO (``genesis/training/train_phase2_rl.py:40-276``).

Objective per step: ``(1 - rl_mix) · NTP + rl_mix · GRPO``.  Both terms go
through ONE backward in the orchestrator (gradient accumulation, clipping and
the optimizer step at the accumulation boundary), so the optimizer sees the
mixed gradient.  The reference backpropagates only the NTP share and leaves
the GRPO term to a separate optimizer call inside the GRPO step.
"""

from __future__ import annotations

import logging
import math
import os
import time
from typing import Any, Callable, Dict, List

import torch
import torch.nn as nn

from genesis.training.grpo import GRPOConfig, GRPOTrainer
from llm_research_b200.ops.loss import shifted_cross_entropy
from olympus.core.training_context import TrainingContext
from olympus.core.training_orchestrator import ModelConfig, ObjectiveConfig, TrainingOrchestrator

logger = logging.getLogger(__name__)


def _ntp_loss(model: nn.Module, input_ids: torch.Tensor):
    out = model(input_ids)
    loss = shifted_cross_entropy(out["logits"], input_ids, ignore_index=-100)
    aux = out.get("aux_loss", 0.0)
    if isinstance(aux, torch.Tensor):
        loss = loss + aux.to(loss.dtype)
    elif isinstance(aux, (int, float)) and aux > 0:
        loss = loss + aux
    v = float(loss.detach())
    return loss, (min(math.exp(v), 1e6) if v < 20 else 1e6)


class RLPretrainer:
    def __init__(self, model: nn.Module, ref_model: nn.Module, reward_fn: Callable[[str, str], float], optimizer,
                 config: dict) -> None:
        self.config = config
        self.device = torch.device(config.get("device", "cuda"))
        self.model = model.to(self.device)
        self.ref_model = ref_model.to(self.device)
        self.optimizer = optimizer
        self.reward_fn = reward_fn
        self.ref_model.eval()
        for p in self.ref_model.parameters():
            p.requires_grad = False
        self.rl_mix = float(config.get("rl_mix", 0.2))
        self.ntp_mix = 1.0 - self.rl_mix
        self.grpo = GRPOTrainer(self.model, self.ref_model, self.reward_fn, GRPOConfig(
            group_size=config.get("grpo_group_size", 8), kl_coeff=config.get("grpo_kl_coeff", 0.1),
            clip_range=config.get("grpo_clip_range", 0.2), max_completion_tokens=config.get("grpo_max_tokens", 256)))
        self.orchestrator = TrainingOrchestrator(gradient_accumulation_steps=config.get("gradient_accumulation_steps", 4),
                                                 device=self.device)
        self.orchestrator.add_model(ModelConfig(name="hlrt", model=self.model, optimizer=self.optimizer,
                                                max_grad_norm=config.get("max_grad_norm", 1.0),
                                                enabled_phases=["rl_pretrain"]))
        self._last: Dict[str, float] = {}
        self.orchestrator.add_objective(ObjectiveConfig(name="ntp", compute_fn=self._ntp_objective, weight=self.ntp_mix,
                                                        enabled_phases=["rl_pretrain"]))
        self.orchestrator.add_objective(ObjectiveConfig(name="grpo", compute_fn=self._grpo_objective,
                                                        weight=self.rl_mix, enabled_phases=["rl_pretrain"]))
        self.orchestrator.set_phase("rl_pretrain")
        self._reward_history: List[float] = []
        self._step_count = 0

    def _ntp_objective(self, models: Dict[str, nn.Module], ctx: TrainingContext, batch: Any) -> torch.Tensor:
        loss, ppl = _ntp_loss(models["hlrt"], batch["input_ids"].to(self.device, non_blocking=True))
        self._last["perplexity"] = ppl
        return loss

    def _grpo_objective(self, models: Dict[str, nn.Module], ctx: TrainingContext, batch: Any) -> torch.Tensor:
        if self.rl_mix <= 0 or "prompts" not in batch:
            self._last.update(loss=0.0, reward_mean=0.0, reward_std=0.0)
            return torch.zeros((), device=self.device)
        loss, metrics = self.grpo.batch_loss(batch)
        self._last.update(metrics)
        return loss

    def train_step(self, batch: Dict[str, Any]) -> Dict[str, float]:
        self.model.train()
        losses = self.orchestrator.step(batch)
        ntp = float(losses["ntp"])
        rl = float(self._last.get("loss", 0.0))
        reward = float(self._last.get("reward_mean", 0.0))
        self._reward_history.append(reward)
        self._step_count += 1
        return {"ntp_loss": ntp, "rl_loss": rl, "total_loss": self.ntp_mix * ntp + self.rl_mix * rl,
                "perplexity": self._last.get("perplexity", float("inf")), "avg_reward": reward,
                "reward_std": float(self._last.get("reward_std", 0.0))}

    def train_epoch(self, dataloader) -> Dict[str, float]:
        tot_ntp = tot_rl = tot_r = 0.0
        n = 0
        log_interval = self.config.get("log_interval", 100)
        save_interval = self.config.get("save_interval", 5000)
        ckpt_dir = self.config.get("checkpoint_dir", "checkpoints/phase2")
        t0 = time.time()
        for batch in dataloader:
            m = self.train_step(batch)
            tot_ntp += m["ntp_loss"]
            tot_rl += m["rl_loss"]
            tot_r += m["avg_reward"]
            n += 1
            step = self.orchestrator.global_step
            if n % log_interval == 0:
                logger.info("Step %d | ntp=%.4f | rl=%.4f | ppl=%.2f | reward=%.4f +/- %.4f", step, m["ntp_loss"],
                            m["rl_loss"], m["perplexity"], m["avg_reward"], m["reward_std"])
            if save_interval > 0 and step > 0 and step % save_interval == 0:
                os.makedirs(ckpt_dir, exist_ok=True)
                self.orchestrator.save_checkpoint(os.path.join(ckpt_dir, f"checkpoint_step{step}.pt"))
        n = max(n, 1)
        avg = tot_ntp / n
        logger.info("Phase 2 epoch done in %.1fs", time.time() - t0)
        return {"epoch_ntp_loss": avg, "epoch_rl_loss": tot_rl / n,
                "epoch_perplexity": min(math.exp(avg), 1e6) if avg < 20 else 1e6,
                "epoch_avg_reward": tot_r / n, "total_steps": n}
