"""Token-level corruptions for verifier negatives (``genesis/verifier/negative_generator.py:17-323``).

Each strategy takes a 1-D id tensor and returns ``(corrupted_ids, labels,
locations)``; ``labels`` is 1.0 on clean positions and 0.0 on corrupted ones.

* ``entity_swap``: 5–15 % of positions get a different uniform token;
* ``negation_insertion``: with existing negation tokens, 50 % chance to delete
  them all; otherwise insert 1–3 negation tokens (``≤ len // 10``);
* ``number_perturbation``: 3–8 % of positions move by ±(10–50 %) of their id
  (±1–10 when that rounds to 0), clamped to the vocabulary, never unchanged;
* ``fact_substitution``: 1–3 spans (``≤ len // 20``) of 2–5 random tokens;
* ``temporal_shift``: swap known temporal marker pairs, else ``entity_swap``.

The token-id heuristics (negation ids, temporal pairs) are the reference's
defaults and are overridable.  Work is done on a host copy with vectorised
tensor ops; results return on the input's device.  Randomness comes from
Python's ``random`` module, so ``random.seed`` makes runs repeatable.
"""

from __future__ import annotations

import random
from typing import Callable, Dict, List, Optional, Tuple

import torch

DEFAULT_CORRUPTION_TYPES: List[str] = ["entity_swap", "negation_insertion", "number_perturbation",
                                       "fact_substitution", "temporal_shift"]
_NEGATION_TOKENS: List[int] = [451, 694, 1790, 3782]
_TEMPORAL_TOKENS: Dict[int, int] = {8091: 10643, 10643: 8091, 1434: 1156, 1156: 1434, 4940: 5765, 5765: 4940}

Result = Tuple[torch.Tensor, torch.Tensor, List[int]]


class NegativeGenerator:
    def __init__(self, corruption_types: Optional[List[str]] = None, vocab_size: int = 32000,
                 negation_tokens: Optional[List[int]] = None, temporal_map: Optional[Dict[int, int]] = None) -> None:
        self.corruption_types = corruption_types or list(DEFAULT_CORRUPTION_TYPES)
        self.vocab_size = vocab_size
        self.negation_tokens = negation_tokens or list(_NEGATION_TOKENS)
        self.temporal_map = temporal_map or dict(_TEMPORAL_TOKENS)
        self._dispatch: Dict[str, Callable[[torch.Tensor], Result]] = {
            "entity_swap": self.entity_swap,
            "negation_insertion": self.negation_insertion,
            "number_perturbation": self.number_perturbation,
            "fact_substitution": self.fact_substitution,
            "temporal_shift": self.temporal_shift,
        }

    # ------------------------------------------------------------------ API
    def corrupt(self, input_ids: torch.Tensor, corruption_type: Optional[str] = None) -> Result:
        kind = corruption_type if corruption_type is not None else random.choice(self.corruption_types)
        fn = self._dispatch.get(kind)
        if fn is None:
            raise ValueError(f"Unknown corruption type '{kind}'. Available: {list(self._dispatch)}")
        return fn(input_ids)

    def batch_corrupt(self, input_ids_batch: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Corrupt each row; pad to the longest result (ids 0, labels 1.0)."""
        host = input_ids_batch.detach().cpu()
        outs = [self.corrupt(host[i])[:2] for i in range(host.size(0))]
        width = max(ids.numel() for ids, _ in outs)
        ids_b = torch.zeros(len(outs), width, dtype=torch.long)
        lab_b = torch.ones(len(outs), width, dtype=torch.float)
        for i, (ids, lab) in enumerate(outs):
            ids_b[i, :ids.numel()] = ids
            lab_b[i, :lab.numel()] = lab
        dev = input_ids_batch.device
        return ids_b.to(dev, non_blocking=True), lab_b.to(dev, non_blocking=True)

    # ------------------------------------------------------------ helpers
    @staticmethod
    def _host(input_ids: torch.Tensor) -> torch.Tensor:
        return input_ids.detach().to("cpu", torch.long).clone()

    @staticmethod
    def _back(ids: torch.Tensor, labels: torch.Tensor, like: torch.Tensor, locs: List[int]) -> Result:
        return ids.to(like.device), labels.to(like.device), locs

    # ----------------------------------------------------------- strategies
    def entity_swap(self, input_ids: torch.Tensor) -> Result:
        ids = self._host(input_ids)
        n = ids.numel()
        k = min(max(1, int(n * random.uniform(0.05, 0.15))), n)
        pos = random.sample(range(n), k)
        p = torch.tensor(pos, dtype=torch.long)
        # a uniform token different from the original: shift by 1..V-1 modulo V
        shift = torch.tensor([random.randint(1, self.vocab_size - 1) for _ in pos], dtype=torch.long)
        ids[p] = (ids[p] + shift) % self.vocab_size
        labels = torch.ones(n)
        labels[p] = 0.0
        return self._back(ids, labels, input_ids, pos)

    def negation_insertion(self, input_ids: torch.Tensor) -> Result:
        ids = self._host(input_ids)
        n = ids.numel()
        is_neg = torch.isin(ids, torch.tensor(self.negation_tokens, dtype=torch.long))
        neg_pos = is_neg.nonzero().flatten().tolist()
        if neg_pos and random.random() < 0.5:
            keep = ~is_neg
            return self._back(ids[keep], torch.ones(int(keep.sum())), input_ids, list(reversed(neg_pos)))
        count = random.randint(1, min(3, max(1, n // 10)))
        at = sorted(random.sample(range(n), min(count, n)), reverse=True)
        out, lab = ids.tolist(), [1.0] * n
        for p in at:
            out.insert(p, random.choice(self.negation_tokens))
            lab.insert(p, 0.0)
        return self._back(torch.tensor(out, dtype=torch.long), torch.tensor(lab), input_ids, at)

    def number_perturbation(self, input_ids: torch.Tensor) -> Result:
        ids = self._host(input_ids)
        n = ids.numel()
        k = min(max(1, int(n * random.uniform(0.03, 0.08))), n)
        pos = random.sample(range(n), k)
        labels = torch.ones(n)
        for p in pos:
            orig = int(ids[p])
            delta = int(orig * random.uniform(0.1, 0.5)) or random.randint(1, 10)
            if random.random() < 0.5:
                delta = -delta
            new = max(0, min(self.vocab_size - 1, orig + delta))
            ids[p] = new if new != orig else (orig + 1) % self.vocab_size
            labels[p] = 0.0
        return self._back(ids, labels, input_ids, pos)

    def fact_substitution(self, input_ids: torch.Tensor) -> Result:
        ids = self._host(input_ids)
        n = ids.numel()
        labels = torch.ones(n)
        locs: List[int] = []
        for _ in range(random.randint(1, min(3, max(1, n // 20)))):
            span = random.randint(2, min(5, n)) if n >= 2 else n
            start = random.randint(0, max(0, n - span))
            stop = min(start + span, n)
            ids[start:stop] = torch.randint(0, self.vocab_size, (stop - start,),
                                            generator=torch.Generator().manual_seed(random.getrandbits(63)))
            labels[start:stop] = 0.0
            locs.extend(range(start, stop))
        return self._back(ids, labels, input_ids, locs)

    def temporal_shift(self, input_ids: torch.Tensor) -> Result:
        ids = self._host(input_ids)
        keys = torch.tensor(list(self.temporal_map), dtype=torch.long)
        hit = torch.isin(ids, keys)
        if not bool(hit.any()):
            return self.entity_swap(input_ids)
        pos = hit.nonzero().flatten()
        ids[pos] = torch.tensor([self.temporal_map[int(t)] for t in ids[pos]], dtype=torch.long)
        labels = torch.ones(ids.numel())
        labels[pos] = 0.0
        return self._back(ids, labels, input_ids, pos.tolist())
