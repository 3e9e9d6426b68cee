"""ACT-V: adversarial co-training of generator and verifier (``genesis/training/train_actv.py:41-449``).

* Verifier step: BCE of all four heads on real text (label 1), on the same
  batch corrupted by ``NegativeGenerator`` (label 0) and, once the replay
  buffer holds ``replay_min_size`` entries, on replayed generator outputs
  against their stored scores; the mean of the active terms is minimised
  with the verifier's AdamW (clip ``max_grad_norm``).
* Generator step: NTP on ``labels`` plus ``alpha · (1 - V.overall)`` where the
  verifier term is computed without gradient (it shifts the reported loss,
  not the update, exactly as in the reference); every sequence is pushed to
  the replay buffer with its scores.
* Every ``distill_interval`` steps: MSE between the projected mean hidden
  states of generator and verifier on up to 32 replayed sequences.

Work layout: real and corrupted rows of equal length share one verifier
forward; replay entries are written with one device→host copy per batch.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Any, Dict, Optional

import torch
import torch.nn as nn

from genesis.verifier.distillation import VerificationDistillation
from genesis.verifier.negative_generator import NegativeGenerator
from genesis.verifier.replay_buffer import ReplayBuffer
from genesis.verifier.verification_head import VerificationHead
from genesis.verifier.verifier_model import VerifierModel
from llm_research_b200.ops.loss import shifted_cross_entropy
from olympus.core.training_orchestrator import ModelConfig, TrainingOrchestrator

logger = logging.getLogger(__name__)

_HEADS = ("factual_score", "logical_score", "stylistic_score")


@dataclass
class ACTVConfig:
    alpha: float = 0.1
    distill_interval: int = 1000
    replay_max_size: int = 10_000
    replay_min_size: int = 100
    replay_batch_ratio: float = 0.25
    distillation_shared_dim: int = 256
    distillation_alpha: float = 0.5
    verifier_lr_mult: float = 1.0
    gradient_accumulation_steps: int = 1
    max_grad_norm: float = 1.0
    device: str = "cpu"


def _get_hidden_dim(model: nn.Module) -> int:
    for attr in ("d_model", "hidden_size", "config"):
        if hasattr(model, attr):
            val = getattr(model, attr)
            if isinstance(val, int):
                return val
            for inner in ("d_model", "hidden_size"):
                if hasattr(val, inner):
                    return int(getattr(val, inner))
    raise ValueError(f"Cannot infer the hidden size of {type(model).__name__}")


def _fit(ids: torch.Tensor, width: int) -> torch.Tensor:
    if ids.size(1) >= width:
        return ids[:, :width]
    return torch.cat([ids, ids.new_zeros(ids.size(0), width - ids.size(1))], dim=1)


class ACTVTrainer:
    def __init__(self, generator: nn.Module, verifier: VerifierModel, neg_generator: NegativeGenerator,
                 replay_buffer: ReplayBuffer, config: ACTVConfig) -> None:
        self.config = config
        self.device = torch.device(config.device)
        self.generator = generator.to(self.device)
        self.verifier = verifier.to(self.device)
        self.neg_generator = neg_generator
        self.replay_buffer = replay_buffer
        self.verification_head = VerificationHead(d_model=verifier.d_model).to(self.device)
        self.distillation = VerificationDistillation(_get_hidden_dim(generator), verifier.d_model,
                                                     shared_dim=config.distillation_shared_dim,
                                                     alpha=config.distillation_alpha).to(self.device)
        self.generator_optimizer = torch.optim.AdamW(self.generator.parameters(), lr=3e-4, weight_decay=0.01)
        self._v_params = list(self.verifier.parameters()) + list(self.verification_head.parameters())
        self.verifier_optimizer = torch.optim.AdamW(self._v_params, lr=3e-4 * config.verifier_lr_mult,
                                                    weight_decay=0.01)
        self.orchestrator = TrainingOrchestrator(gradient_accumulation_steps=config.gradient_accumulation_steps,
                                                 device=self.device)
        self.orchestrator.add_model(ModelConfig(name="generator", model=self.generator,
                                                optimizer=self.generator_optimizer, max_grad_norm=config.max_grad_norm))
        self.orchestrator.add_model(ModelConfig(name="verifier", model=self.verifier,
                                                optimizer=self.verifier_optimizer, max_grad_norm=config.max_grad_norm))
        self._step_count = 0

    def _score(self, ids: torch.Tensor) -> Dict[str, torch.Tensor]:
        return self.verification_head(self.verifier(ids)["pooled_output"])

    # -------------------------------------------------------------- verifier
    def train_verifier_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, float]:
        ids = batch["input_ids"].to(self.device, non_blocking=True)
        B = ids.size(0)
        self.verifier.train()
        self.verification_head.train()
        bad, _ = self.neg_generator.batch_corrupt(ids)
        bad = bad.to(self.device, non_blocking=True)
        if bad.size(1) == ids.size(1):
            s = self._score(torch.cat([ids, bad]))
            pos = {k: v[:B] for k, v in s.items()}
            neg = {k: v[B:] for k, v in s.items()}
        else:
            pos, neg = self._score(ids), self._score(bad)
        pos_loss = self.verification_head.compute_loss(pos, {k: torch.ones_like(v) for k, v in pos.items()})
        neg_loss = self.verification_head.compute_loss(neg, {k: torch.zeros_like(v) for k, v in neg.items()})
        replay_loss = torch.zeros((), device=self.device)
        terms = 2.0
        if self.replay_buffer.is_ready(self.config.replay_min_size):
            samples = self.replay_buffer.sample(max(1, int(B * self.config.replay_batch_ratio)))
            if samples:
                r_ids = _fit(torch.stack([s["input_ids"] for s in samples]), ids.size(1)).to(self.device)
                r_scores = self._score(r_ids)
                labels = {k: torch.stack([s["scores"][k] for s in samples]).to(self.device) for k in _HEADS}
                replay_loss = self.verification_head.compute_loss(r_scores, labels)
                terms = 3.0
        total = (pos_loss + neg_loss + replay_loss) / terms
        self.verifier_optimizer.zero_grad(set_to_none=True)
        total.backward()
        nn.utils.clip_grad_norm_(self._v_params, self.config.max_grad_norm)
        self.verifier_optimizer.step()
        h = torch.stack([pos_loss.detach(), neg_loss.detach(), replay_loss.detach(), total.detach()]).tolist()
        return {"pos_loss": h[0], "neg_loss": h[1], "replay_loss": h[2], "verifier_loss": h[3]}

    # ------------------------------------------------------------- generator
    def train_generator_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, Any]:
        ids = batch["input_ids"].to(self.device, non_blocking=True)
        labels = batch.get("labels", batch["input_ids"]).to(self.device, non_blocking=True)
        self.generator.train()
        out = self.generator(ids)
        logits = out["logits"] if isinstance(out, dict) else out
        ntp = shifted_cross_entropy(logits, labels, ignore_index=-100)
        with torch.no_grad():
            v_scores = self._score(ids)
            feedback = (1.0 - v_scores["overall_score"]).mean()
        self.replay_buffer.add_batch(ids, v_scores, metadata={"step": self._step_count})
        total = ntp + self.config.alpha * feedback
        self.generator_optimizer.zero_grad(set_to_none=True)
        total.backward()
        nn.utils.clip_grad_norm_(self.generator.parameters(), self.config.max_grad_norm)
        self.generator_optimizer.step()
        keys = list(v_scores)
        h = torch.stack([ntp.detach().float(), feedback.float(), total.detach().float()]
                        + [v_scores[k].float().mean() for k in keys]).tolist()
        return {"ntp_loss": h[0], "feedback_loss": h[1], "generator_loss": h[2],
                "v_scores": {k: h[3 + i] for i, k in enumerate(keys)}}

    # ------------------------------------------------------------ co-training
    def co_training_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, Any]:
        v = self.train_verifier_step(batch)
        g = self.train_generator_step(batch)
        self._step_count += 1
        metrics: Dict[str, Any] = {**{f"v_{k}": x for k, x in v.items()}, **{f"g_{k}": x for k, x in g.items()},
                                   "step": self._step_count}
        if self._step_count % self.config.distill_interval == 0:
            loss = self._distill()
            if loss is not None:
                metrics["distillation_loss"] = loss
        return metrics

    def _distill(self) -> Optional[float]:
        if not self.replay_buffer.is_ready(self.config.replay_min_size):
            return None
        samples = self.replay_buffer.sample(min(32, self.replay_buffer.size))
        if not samples:
            return None
        width = max(s["input_ids"].numel() for s in samples)
        ids = torch.stack([_fit(s["input_ids"].view(1, -1), width)[0] for s in samples]).to(self.device)
        self.generator.train()
        out = self.generator(ids)
        g_hidden = out.get("hidden_states", out["logits"]) if isinstance(out, dict) else out
        with torch.no_grad():
            v_hidden = self.verifier(ids)["hidden_states"]
        g = g_hidden.mean(dim=1) if g_hidden.dim() == 3 else g_hidden
        vh = v_hidden.mean(dim=1) if v_hidden.dim() == 3 else v_hidden
        loss = self.distillation(g.float(), vh.float())
        self.generator_optimizer.zero_grad(set_to_none=True)
        loss.backward()
        nn.utils.clip_grad_norm_(self.generator.parameters(), self.config.max_grad_norm)
        self.generator_optimizer.step()
        return float(loss.detach())

    def save_checkpoint(self, path: str) -> None:
        self.orchestrator.save_checkpoint(path)

    def load_checkpoint(self, path: str) -> None:
        self.orchestrator.load_checkpoint(path)
