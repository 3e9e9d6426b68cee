"""Replay memory of past generator outputs for the ACT-V verifier
(reference: ``genesis/verifier/replay_buffer.py:16-123``).

Behaviour kept from the reference: entries are ``{"input_ids", "scores",
"metadata"}`` held on the host, the capacity is ``max_size`` entries with the
oldest overwritten first, ``sample(n)`` returns ``min(n, size)`` distinct
entries drawn uniformly, and ``is_ready(min_size)`` gates replay.

Layout.  Writes go to slot ``written % max_size`` of a fixed slot table, where
``written`` counts every entry ever added, so the ring needs no separate write
pointer and ``size == min(written, max_size)``.  A slot holds a reference to a
host batch and a row index rather than a copy of the row: ``add_batch`` moves
a whole generated batch (token ids and every score tensor) to the host with
one copy each and fills ``B`` slots with row references, and a sampled entry
is materialised as row views of those batches.  Sampling draws a permutation
prefix with a torch generator seeded from Python's ``random`` module, so
``random.seed`` makes it reproducible as before.
"""

from __future__ import annotations

import random
from typing import Any, Dict, List, Optional, Tuple

import torch

_Slot = Tuple[torch.Tensor, Dict[str, torch.Tensor], Dict[str, Any], int]  # ids, scores, metadata, row


class ReplayBuffer:
    def __init__(self, max_size: int = 10000) -> None:
        if max_size <= 0:
            raise ValueError(f"ReplayBuffer capacity must be a positive number of entries, not {max_size}")
        self.max_size = int(max_size)
        self._slots: List[Optional[_Slot]] = [None] * self.max_size
        self._written = 0

    # ----------------------------------------------------------------- size
    @property
    def size(self) -> int:
        return min(self._written, self.max_size)

    def __len__(self) -> int:
        return self.size

    def is_ready(self, min_size: int = 100) -> bool:
        return self.size >= min_size

    # --------------------------------------------------------------- writes
    def _put(self, ids: torch.Tensor, scores: Dict[str, torch.Tensor], metadata: Dict[str, Any], row: int) -> None:
        self._slots[self._written % self.max_size] = (ids, scores, metadata, row)
        self._written += 1

    def add(self, input_ids: torch.Tensor, scores: Dict[str, torch.Tensor],
            metadata: Optional[Dict[str, Any]] = None) -> None:
        """Store one sequence (any shape) with its per-head scores."""
        ids = input_ids.detach().to("cpu").unsqueeze(0)
        host = {k: v.detach().to("cpu").unsqueeze(0) for k, v in scores.items()}
        self._put(ids, host, dict(metadata or {}), 0)

    def add_batch(self, input_ids: torch.Tensor, scores: Dict[str, torch.Tensor],
                  metadata: Optional[Dict[str, Any]] = None) -> None:
        """Store every row of a ``(B, S)`` batch: one device-to-host copy per tensor,
        ``B`` slots referencing rows of the host batch."""
        ids = input_ids.detach().to("cpu")
        host = {k: v.detach().to("cpu") for k, v in scores.items()}
        meta = dict(metadata or {})
        for r in range(ids.shape[0]):
            self._put(ids, host, meta, r)

    # ---------------------------------------------------------------- reads
    @staticmethod
    def _entry(slot: _Slot) -> Dict[str, Any]:
        ids, scores, meta, r = slot
        return {"input_ids": ids[r], "scores": {k: v[r] for k, v in scores.items()}, "metadata": meta}

    def sample(self, batch_size: int) -> List[Dict[str, Any]]:
        n = self.size
        k = min(int(batch_size), n)
        if k <= 0:
            return []
        gen = torch.Generator().manual_seed(random.getrandbits(63))
        picks = torch.randperm(n, generator=gen)[:k].tolist()
        return [self._entry(self._slots[i]) for i in picks]

    def clear(self) -> None:
        self._slots = [None] * self.max_size
        self._written = 0

    def __repr__(self) -> str:
        return f"ReplayBuffer({self.size}/{self.max_size} entries, written={self._written})"
