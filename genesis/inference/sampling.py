"""Next-token sampling (``genesis/inference/sampling.py:16-146``).

Order of application in :func:`sample`: repetition penalty (HF rule: divide
positive, multiply negative scores of already generated ids), temperature,
greedy arg-max when ``temperature <= 0``, top-k, top-p (smallest prefix of the
sorted distribution whose mass before the token is below ``p``), multinomial.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F


@dataclass
class SamplingConfig:
    temperature: float = 1.0
    top_k: int = 50
    top_p: float = 0.9
    repetition_penalty: float = 1.0
    min_tokens: int = 0


def apply_temperature(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    if temperature == 1.0 or temperature <= 0.0:
        return logits
    return logits / temperature


def apply_top_k(logits: torch.Tensor, k: int) -> torch.Tensor:
    if k <= 0 or k >= logits.size(-1):
        return logits
    kth = torch.topk(logits, k, dim=-1).values[..., -1:]
    return logits.masked_fill(logits < kth, float("-inf"))


def apply_top_p(logits: torch.Tensor, p: float) -> torch.Tensor:
    if p >= 1.0:
        return logits
    sorted_logits, order = torch.sort(logits, descending=True, dim=-1)
    probs = F.softmax(sorted_logits, dim=-1)
    mass_before = torch.cumsum(probs, dim=-1) - probs
    sorted_logits = sorted_logits.masked_fill(mass_before >= p, float("-inf"))
    return torch.empty_like(logits).scatter_(-1, order, sorted_logits)


def apply_repetition_penalty(logits: torch.Tensor, generated_ids: torch.Tensor, penalty: float) -> torch.Tensor:
    if penalty == 1.0:
        return logits
    seen = torch.gather(logits, -1, generated_ids)
    seen = torch.where(seen > 0, seen / penalty, seen * penalty)
    return logits.scatter(-1, generated_ids, seen)


def sample(logits: torch.Tensor, config: SamplingConfig, generated_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
    if generated_ids is not None and config.repetition_penalty != 1.0:
        logits = apply_repetition_penalty(logits, generated_ids, config.repetition_penalty)
    logits = apply_temperature(logits, config.temperature)
    if config.temperature <= 0.0:
        return logits.argmax(dim=-1)
    logits = apply_top_p(apply_top_k(logits, config.top_k), config.top_p)
    return torch.multinomial(F.softmax(logits.float(), dim=-1), num_samples=1).squeeze(-1)
