"""Group Relative Policy Optimisation (``genesis/training/grpo.py:26-303``).

Per prompt, ``G`` completions are sampled; rewards are z-scored inside the
group (std clamped to ``min_group_std``) to give advantages; the loss is the
PPO-clipped surrogate on the sequence log-prob ratio against the frozen
reference policy plus ``kl_coeff`` × Schulman's approximate KL
``(r - 1) - log r``.

B200 shape of the work: the ``G`` completions of a prompt are sampled as ONE
batch with the KV cache (``genesis.inference.Generator``) instead of a full
re-forward per token per completion, and their log-probs under the policy and
the reference come from ONE padded forward each per prompt group.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from genesis.training.reward_functions import completion_logprobs, encode_ids


@dataclass
class GRPOConfig:
    group_size: int = 8
    kl_coeff: float = 0.1
    clip_range: float = 0.2
    temperature: float = 1.0
    max_completion_tokens: int = 256
    min_group_std: float = 1e-8


def _eos_id(tokenizer: Any) -> Optional[int]:
    eos = getattr(tokenizer, "eos_token_id", None)
    return int(eos) if eos is not None else None


def _decode(tokenizer: Any, ids: Sequence[int]) -> str:
    try:
        return tokenizer.decode(list(ids), skip_special_tokens=True)
    except TypeError:
        return tokenizer.decode(list(ids))


@torch.no_grad()
def sample_group(model: nn.Module, prompt_ids: Sequence[int], group_size: int, max_new_tokens: int,
                 temperature: float, eos_id: Optional[int], device: torch.device) -> List[List[int]]:
    """``group_size`` sampled continuations of one prompt, each cut after its first EOS."""
    from genesis.model.hlrt import HLRT

    ids = torch.tensor([list(prompt_ids)] * group_size, dtype=torch.long, device=device)
    if isinstance(model, HLRT):
        from genesis.inference.generator import GenerationConfig, Generator
        from genesis.inference.sampling import SamplingConfig

        cfg = GenerationConfig(max_new_tokens=max_new_tokens, eos_token_id=eos_id,
                               sampling=SamplingConfig(temperature=max(temperature, 1e-8)))
        new = Generator(model).generate(ids, cfg)["new_token_ids"]
    else:
        steps = []
        seq = ids
        for _ in range(max_new_tokens):
            logits = model(seq)["logits"][:, -1, :].float() / max(temperature, 1e-8)
            tok = torch.multinomial(F.softmax(logits, dim=-1), 1)
            steps.append(tok)
            seq = torch.cat([seq, tok], dim=1)
            if eos_id is not None and bool((torch.cat(steps, 1) == eos_id).any(dim=1).all()):
                break
        new = torch.cat(steps, dim=1) if steps else ids[:, :0]
    out = []
    for row in new.tolist():
        if eos_id is not None and eos_id in row:
            row = row[:row.index(eos_id) + 1]
        out.append(row)
    return out


class GRPOTrainer:
    def __init__(self, model: nn.Module, ref_model: nn.Module, reward_fn: Callable[[str, str], float],
                 config: Optional[GRPOConfig] = None) -> None:
        self.model = model
        self.ref_model = ref_model
        self.reward_fn = reward_fn
        self.config = config or GRPOConfig()
        self.ref_model.eval()
        for p in self.ref_model.parameters():
            p.requires_grad = False

    # ------------------------------------------------------------ sampling
    @torch.no_grad()
    def generate_group_ids(self, prompts: List[str], tokenizer: Any) -> Tuple[List[List[int]], List[List[List[int]]]]:
        was_training = self.model.training
        self.model.eval()
        device = next(self.model.parameters()).device
        prompt_ids = [encode_ids(tokenizer, p) for p in prompts]
        groups = [sample_group(self.model, ids, self.config.group_size, self.config.max_completion_tokens,
                               self.config.temperature, _eos_id(tokenizer), device) for ids in prompt_ids]
        self.model.train(was_training)
        return prompt_ids, groups

    @torch.no_grad()
    def generate_group(self, prompts: List[str], tokenizer: Any) -> List[List[str]]:
        _, groups = self.generate_group_ids(prompts, tokenizer)
        return [[_decode(tokenizer, c) for c in g] for g in groups]

    # ---------------------------------------------------------------- math
    def compute_advantages(self, rewards_per_group: torch.Tensor) -> torch.Tensor:
        mean = rewards_per_group.mean(dim=1, keepdim=True)
        std = rewards_per_group.std(dim=1, keepdim=True).clamp(min=self.config.min_group_std)
        return (rewards_per_group - mean) / std

    def compute_loss(self, logprobs: torch.Tensor, ref_logprobs: torch.Tensor,
                     advantages: torch.Tensor) -> Tuple[torch.Tensor, Dict[str, float]]:
        log_ratio = logprobs - ref_logprobs
        ratio = torch.exp(log_ratio)
        eps = self.config.clip_range
        policy_loss = -torch.min(ratio * advantages, ratio.clamp(1.0 - eps, 1.0 + eps) * advantages).mean()
        approx_kl = (ratio - 1.0) - log_ratio
        kl = approx_kl.mean()
        total = policy_loss + self.config.kl_coeff * kl
        stats = torch.stack([policy_loss.detach(), kl.detach(), ((ratio - 1.0).abs() > eps).float().mean(),
                             ratio.detach().mean()]).tolist()  # one device→host read
        return total, {"policy_loss": stats[0], "kl_penalty": stats[1], "kl_div": stats[1],
                       "clip_fraction": stats[2], "mean_ratio": stats[3]}

    # ---------------------------------------------------------------- step
    def sequence_logprobs(self, prompt_ids: List[List[int]], groups: List[List[List[int]]]
                          ) -> Tuple[torch.Tensor, torch.Tensor]:
        """(B, G) summed completion log-probs under the policy (with grad) and the reference."""
        device = next(self.model.parameters()).device
        pol, ref = [], []
        for ids, comps in zip(prompt_ids, groups):
            pre = [ids] * len(comps)
            pol.append(completion_logprobs(self.model, pre, comps, device)[0])
            with torch.no_grad():
                ref.append(completion_logprobs(self.ref_model, pre, comps, device)[0])
        return torch.stack(pol), torch.stack(ref)

    def batch_loss(self, batch: Dict[str, Any]) -> Tuple[torch.Tensor, Dict[str, float]]:
        """Sample, score and return ``(loss, metrics)`` without stepping an optimizer."""
        prompts, tokenizer = batch["prompts"], batch["tokenizer"]
        device = next(self.model.parameters()).device
        prompt_ids, groups = self.generate_group_ids(prompts, tokenizer)
        texts = [[_decode(tokenizer, c) for c in g] for g in groups]
        flat_p = [p for p, g in zip(prompts, texts) for _ in g]
        flat_c = [c for g in texts for c in g]
        scorer = getattr(self.reward_fn, "score_batch", None)
        flat_r = scorer(flat_p, flat_c) if scorer is not None else [self.reward_fn(p, c) for p, c in zip(flat_p, flat_c)]
        rewards = torch.tensor(flat_r, dtype=torch.float32, device=device).view(len(prompts), -1)
        advantages = self.compute_advantages(rewards)
        self.model.train()
        logprobs, ref_logprobs = self.sequence_logprobs(prompt_ids, groups)
        loss, stats = self.compute_loss(logprobs, ref_logprobs, advantages)
        host = torch.stack([loss.detach(), rewards.mean(), rewards.std(), rewards.max(), rewards.min(),
                            advantages.mean(), advantages.std()]).tolist()
        return loss, {"loss": host[0], "reward_mean": host[1], "reward_std": host[2], "reward_max": host[3],
                      "reward_min": host[4], "advantage_mean": host[5], "advantage_std": host[6], **stats}

    def step(self, batch: Dict[str, Any]) -> Dict[str, float]:
        loss, metrics = self.batch_loss(batch)
        if "optimizer" in batch:
            opt = batch["optimizer"]
            opt.zero_grad()
            loss.backward()
            opt.step()
        return metrics
