"""Phase 3: data flywheel on self-generated traces (``genesis/training/train_phase3_flywheel.py:38-325``).

Loop: take the first half (≤ 512 tokens) of each sequence as a context,
sample a trace of ``max_trace_tokens``, score it with
``reward_fn(model, context_ids, trace_ids) -> (B,)``, keep traces at or above
the buffer's threshold in the ``FlywheelBuffer``, and train NTP on a batch in
which ``trace_mix_ratio`` of the rows are replaced by buffered
``context + trace`` sequences.

B200 shape: all contexts of a batch are sampled together with the KV cache
(one batched decode loop, not one re-forward per token per sequence), the
reward is computed for the whole batch in one call, and each stored trace
keeps its token ids in the entry's metadata so mixing does not re-tokenise.
"""

from __future__ import annotations

import logging
from typing import Any, Callable, Dict, List

import torch
import torch.nn as nn

from genesis.training.grpo import sample_group
from llm_research_b200.ops.loss import shifted_cross_entropy
from olympus.core.training_context import TrainingContext
from olympus.core.training_orchestrator import ModelConfig, ObjectiveConfig, TrainingOrchestrator
from olympus.data.flywheel_buffer import FlywheelBuffer
from olympus.data.tokenizer import TokenizerWrapper

logger = logging.getLogger(__name__)


def flywheel_ntp_objective(models: Dict[str, nn.Module], ctx: TrainingContext, batch: Any) -> torch.Tensor:
    model = models["hlrt"]
    ids = batch["input_ids"].to(next(model.parameters()).device, non_blocking=True)
    out = model(ids)
    loss = shifted_cross_entropy(out["logits"], ids, ignore_index=-100)
    aux = out.get("aux_loss", 0.0)
    if isinstance(aux, torch.Tensor):
        loss = loss + aux.to(loss.dtype)
    elif isinstance(aux, (int, float)) and aux > 0:
        loss = loss + aux
    return loss


class FlywheelTrainer:
    def __init__(self, model: nn.Module, flywheel_buffer: FlywheelBuffer, reward_fn: Callable[..., torch.Tensor],
                 optimizer, config: dict) -> None:
        self.config = config
        self.device = torch.device(config.get("device", "cuda"))
        self.model = model.to(self.device)
        self.flywheel_buffer = flywheel_buffer
        self.reward_fn = reward_fn
        self.optimizer = optimizer
        self.reward_threshold = config.get("reward_threshold", 0.1)
        self.trace_mix_ratio = config.get("trace_mix_ratio", 0.3)
        self.generation_interval = config.get("generation_interval", 100)
        self.max_trace_tokens = config.get("max_trace_tokens", 64)
        self.temperature = config.get("temperature", 0.8)
        self.tokenizer = config.get("tokenizer") or TokenizerWrapper(backend=config.get("tokenizer_backend", "tiktoken"),
                                                                    vocab_size=config.get("vocab_size", 32000))
        self.orchestrator = TrainingOrchestrator(gradient_accumulation_steps=config.get("gradient_accumulation_steps", 4),
                                                 device=self.device)
        self.orchestrator.add_model(ModelConfig(name="hlrt", model=self.model, optimizer=self.optimizer,
                                                max_grad_norm=config.get("max_grad_norm", 1.0),
                                                enabled_phases=["flywheel"]))
        self.orchestrator.add_objective(ObjectiveConfig(name="ntp", compute_fn=flywheel_ntp_objective, weight=1.0,
                                                        enabled_phases=["flywheel"]))
        self.orchestrator.set_phase("flywheel")

    @torch.no_grad()
    def generate_traces(self, prompts: List[torch.Tensor]) -> List[Dict[str, Any]]:
        """Sample and score one trace per context; contexts of equal length share one batch."""
        if not prompts:
            return []
        was_training = self.model.training
        self.model.eval()
        results: List[Dict[str, Any]] = [None] * len(prompts)  # type: ignore[list-item]
        by_len: Dict[int, List[int]] = {}
        for i, p in enumerate(prompts):
            by_len.setdefault(int(p.numel()), []).append(i)
        for idxs in by_len.values():
            ctx = torch.stack([prompts[i].to(self.device) for i in idxs])
            gen = sample_group_batch(self.model, ctx, self.max_trace_tokens, self.temperature, self.device)
            reward = self.reward_fn(self.model, ctx, gen)
            if isinstance(reward, torch.Tensor) and reward.numel() == len(idxs):
                rewards = reward.float().flatten().tolist()
            else:  # one scalar for the whole group (a plain float or a 0-d tensor)
                rewards = [float(reward)] * len(idxs)
            ctx_host, gen_host = ctx.cpu(), gen.cpu()
            for j, i in enumerate(idxs):
                results[i] = {"context_ids": ctx_host[j], "trace_ids": gen_host[j], "reward": rewards[j],
                              "context_text": self.tokenizer.decode(ctx_host[j].tolist()),
                              "trace_text": self.tokenizer.decode(gen_host[j].tolist())}
        self.model.train(was_training)
        return results

    def train_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, Any]:
        return self.orchestrator.step(self._mix_with_buffer(batch))

    def flywheel_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, Any]:
        ids = batch["input_ids"]
        ctx_len = max(1, min(ids.shape[1] // 2, 512))
        results = self.generate_traces([row[:ctx_len] for row in ids])
        stored = 0
        for r in results:
            full = torch.cat([r["context_ids"], r["trace_ids"]]).tolist()
            stored += int(self.flywheel_buffer.add(context=r["context_text"], trace=r["trace_text"],
                                                   reward=r["reward"], metadata={"token_ids": full}))
        losses = self.train_step(batch)
        return {"loss": losses.get("total", losses.get("ntp", 0.0)), "traces_generated": len(results),
                "traces_stored": stored, "avg_reward": sum(r["reward"] for r in results) / max(len(results), 1),
                "buffer_size": self.flywheel_buffer.size}

    def _mix_with_buffer(self, batch: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        ids = batch["input_ids"]
        B, S = ids.shape
        if self.flywheel_buffer.size == 0 or self.trace_mix_ratio <= 0:
            return batch
        n = min(max(1, int(B * self.trace_mix_ratio)), self.flywheel_buffer.size, B)
        rows = []
        for entry in self.flywheel_buffer.sample(n):
            toks = entry.get("metadata", {}).get("token_ids")
            if toks is None:
                toks = self.tokenizer.encode(entry["context"] + " " + entry["trace"])
                toks = toks.flatten().tolist() if isinstance(toks, torch.Tensor) else list(toks)
            toks = toks[:S] + [self.tokenizer.pad_id] * max(0, S - len(toks))
            rows.append(toks)
        mixed = ids.clone()
        mixed[:len(rows)] = torch.tensor(rows, dtype=ids.dtype).to(ids.device)
        return {"input_ids": mixed.to(self.device, non_blocking=True)}


@torch.no_grad()
def sample_group_batch(model: nn.Module, ctx: torch.Tensor, max_new_tokens: int, temperature: float,
                       device: torch.device) -> torch.Tensor:
    """(B, T) sampled continuations of a (B, S) batch of equal-length contexts (no EOS stop)."""
    from genesis.model.hlrt import HLRT

    if isinstance(model, HLRT):
        from genesis.inference.generator import GenerationConfig, Generator
        from genesis.inference.sampling import SamplingConfig

        cfg = GenerationConfig(max_new_tokens=max_new_tokens, sampling=SamplingConfig(temperature=max(temperature, 1e-8)))
        return Generator(model).generate(ctx.to(device), cfg)["new_token_ids"]
    rows = [sample_group(model, row.tolist(), 1, max_new_tokens, temperature, None, device)[0] for row in ctx]
    return torch.tensor(rows, dtype=torch.long, device=device)
