"""Reward functions for RL fine-tuning (``genesis/training/reward_functions.py:30-356``).

Every reward maps ``(prompt, completion) -> float``.

* ``InformationGainReward``: ``clamp((ppl_base - ppl_ctx) / ppl_base, min, max)``
  where both perplexities of the completion are measured under a frozen
  reference model, with the prompt and with ``baseline_context``; an empty
  completion scores ``min_reward``.  ``score_batch`` evaluates many pairs in
  two padded forward passes instead of two passes per pair.
* ``CorrectnessReward``: regex answer extraction (``answer is|answer:|=``),
  exact / numeric-tolerance / substring ("partial") match against a table.
* ``FormatReward``: ``<|reason_start|> … <|reason_end|>`` tag pairing plus
  optional regex sections.
* ``CompositeReward``: weighted sum, or weighted mean with ``normalize``.
"""

from __future__ import annotations

import math
import re
from abc import ABC, abstractmethod
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


def encode_ids(tokenizer: Any, text: str) -> List[int]:
    """Token ids of ``text`` from tokenizers that return a list or a tensor."""
    ids = tokenizer.encode(text)
    if isinstance(ids, torch.Tensor):
        ids = ids.flatten().tolist()
    return list(ids)


def completion_logprobs(model: nn.Module, prefixes: Sequence[Sequence[int]], completions: Sequence[Sequence[int]],
                        device: torch.device, pad_id: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-sequence sum and count of completion-token log-probs.

    Rows ``prefix + completion`` of equal length share one forward pass (the
    HLRT tiers pool over the whole sequence, so padding would change the
    result; bucketing by length keeps it exact).  Returns ``(sum, count)`` as
    fp32 tensors of shape ``(N,)``; gradients flow when the model has them.
    """
    n = len(prefixes)
    rows = [list(p) + list(c) for p, c in zip(prefixes, completions)]
    buckets: Dict[int, List[int]] = {}
    for i, r in enumerate(rows):
        buckets.setdefault(len(r), []).append(i)
    sums: List[torch.Tensor] = [torch.zeros((), device=device)] * n
    counts = torch.zeros(n)
    for width, idxs in buckets.items():
        if width < 2:
            continue
        ids = torch.tensor([rows[i] for i in idxs], dtype=torch.long)
        mask = torch.zeros(len(idxs), width - 1)
        for j, i in enumerate(idxs):
            lp_, lc = len(prefixes[i]), len(completions[i])
            # logit position t predicts token t+1: completion tokens sit at [lp_, lp_ + lc)
            lo = max(lp_ - 1, 0)
            mask[j, lo:lp_ + lc - 1] = 1.0
            counts[i] = float(lp_ + lc - 1 - lo)
        ids, mask = ids.to(device), mask.to(device)
        logits = model(ids)["logits"][:, :-1].float()
        lp = F.log_softmax(logits, dim=-1).gather(-1, ids[:, 1:, None]).squeeze(-1)
        tot = (lp * mask).sum(dim=1)
        for j, i in enumerate(idxs):
            sums[i] = tot[j]
    return torch.stack(sums), counts.to(device)


class RewardFunction(ABC):
    @abstractmethod
    def __call__(self, prompt: str, completion: str) -> float:
        ...

    def score_batch(self, prompts: Sequence[str], completions: Sequence[str]) -> List[float]:
        return [self(p, c) for p, c in zip(prompts, completions)]


class InformationGainReward(RewardFunction):
    def __init__(self, ref_model: nn.Module, tokenizer: Any, baseline_context: str = "", max_reward: float = 1.0,
                 min_reward: float = -1.0) -> None:
        self.ref_model = ref_model
        self.tokenizer = tokenizer
        self.baseline_context = baseline_context
        self.max_reward = max_reward
        self.min_reward = min_reward
        self.ref_model.eval()
        for p in self.ref_model.parameters():
            p.requires_grad = False

    def _split(self, context: str, completion: str) -> Tuple[List[int], List[int]]:
        full = encode_ids(self.tokenizer, context + completion)
        n = len(encode_ids(self.tokenizer, context))
        return full[:n], full[n:]

    @torch.no_grad()
    def _perplexities(self, contexts: Sequence[str], completions: Sequence[str]) -> List[float]:
        device = next(self.ref_model.parameters()).device
        pairs = [self._split(c, x) for c, x in zip(contexts, completions)]
        # a completion needs a preceding token to be scored: an empty context scores from its 2nd token
        pre = [p if p else c[:1] for p, c in pairs]
        comp = [c if p else c[1:] for p, c in pairs]
        s, n = completion_logprobs(self.ref_model, pre, comp, device)
        out = []
        for i in range(len(pairs)):
            cnt = float(n[i])
            out.append(1e6 if cnt == 0 else math.exp(-float(s[i]) / cnt))
        return out

    def _compute_perplexity(self, context: str, completion: str) -> float:
        return self._perplexities([context], [completion])[0]

    def _gain(self, base: float, ctx: float) -> float:
        if base < 1e-8:
            return 0.0
        return max(self.min_reward, min(self.max_reward, (base - ctx) / base))

    def __call__(self, prompt: str, completion: str) -> float:
        return self.score_batch([prompt], [completion])[0]

    def score_batch(self, prompts: Sequence[str], completions: Sequence[str]) -> List[float]:
        live = [i for i, c in enumerate(completions) if c.strip()]
        out = [self.min_reward] * len(prompts)
        if live:
            base = self._perplexities([self.baseline_context] * len(live), [completions[i] for i in live])
            ctx = self._perplexities([prompts[i] for i in live], [completions[i] for i in live])
            for j, i in enumerate(live):
                out[i] = self._gain(base[j], ctx[j])
        return out


class CorrectnessReward(RewardFunction):
    def __init__(self, expected_answers: Optional[Dict[str, str]] = None,
                 answer_pattern: str = r"(?:answer is|answer:|=)\s*(?P<answer>[^\n,.]+)",
                 numeric_tolerance: float = 1e-6, correct_reward: float = 1.0, incorrect_reward: float = 0.0,
                 partial_reward: float = 0.5) -> None:
        self.expected_answers = expected_answers or {}
        self.answer_pattern = re.compile(answer_pattern, re.IGNORECASE)
        self.numeric_tolerance = numeric_tolerance
        self.correct_reward = correct_reward
        self.incorrect_reward = incorrect_reward
        self.partial_reward = partial_reward

    def _extract_answer(self, text: str) -> Optional[str]:
        m = self.answer_pattern.search(text)
        return m.group("answer").strip() if m else None

    def _is_numeric_match(self, a: str, b: str) -> bool:
        try:
            return abs(float(a.replace(",", "").strip()) - float(b.replace(",", "").strip())) <= self.numeric_tolerance
        except (ValueError, TypeError):
            return False

    def __call__(self, prompt: str, completion: str) -> float:
        expected = self.expected_answers.get(prompt)
        if expected is None:
            return self.incorrect_reward
        want = expected.strip().lower()
        got = self._extract_answer(completion)
        if got is None:
            return self.partial_reward if want in completion.lower() else self.incorrect_reward
        if got.lower() == want or self._is_numeric_match(got, expected):
            return self.correct_reward
        return self.partial_reward if want in got.lower() else self.incorrect_reward


class FormatReward(RewardFunction):
    def __init__(self, reason_start_tag: str = "<|reason_start|>", reason_end_tag: str = "<|reason_end|>",
                 required_sections: Optional[List[str]] = None, tag_reward: float = 0.5,
                 structure_reward: float = 0.25, max_reward: float = 1.0) -> None:
        self.reason_start_tag = reason_start_tag
        self.reason_end_tag = reason_end_tag
        self.required_sections = required_sections or []
        self.tag_reward = tag_reward
        self.structure_reward = structure_reward
        self.max_reward = max_reward

    def __call__(self, prompt: str, completion: str) -> float:
        if not completion.strip():
            return 0.0
        r = 0.0
        a, b = completion.find(self.reason_start_tag), completion.find(self.reason_end_tag)
        if a >= 0 and b >= 0:
            if b > a:
                inner = completion[a + len(self.reason_start_tag):b]
                r += self.tag_reward if inner.strip() else 0.25 * self.tag_reward
        elif a >= 0 or b >= 0:
            r += 0.1 * self.tag_reward
        if self.required_sections:
            each = self.structure_reward / len(self.required_sections)
            r += each * sum(1 for pat in self.required_sections if re.search(pat, completion, re.IGNORECASE))
        return min(self.max_reward, r)


class CompositeReward(RewardFunction):
    def __init__(self, rewards_and_weights: List[Tuple[RewardFunction, float]], normalize: bool = True) -> None:
        if not rewards_and_weights:
            raise ValueError("Must provide at least one (reward_fn, weight) pair.")
        self.rewards_and_weights = rewards_and_weights
        self.normalize = normalize

    def __call__(self, prompt: str, completion: str) -> float:
        return self.score_batch([prompt], [completion])[0]

    def score_batch(self, prompts: Sequence[str], completions: Sequence[str]) -> List[float]:
        total = [0.0] * len(prompts)
        wsum = 0.0
        for fn, w in self.rewards_and_weights:
            for i, s in enumerate(fn.score_batch(prompts, completions)):
                total[i] += w * s
            wsum += w
        if self.normalize and wsum > 0:
            return [t / wsum for t in total]
        return total
