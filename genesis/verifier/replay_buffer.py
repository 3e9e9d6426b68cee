"""FIFO ring buffer of past generator outputs (``genesis/verifier/replay_buffer.py:16-123``).

Entries are ``{"input_ids", "scores", "metadata"}`` stored detached on the
host; once ``max_size`` entries are held the oldest is overwritten.
``sample(n)`` draws ``min(n, size)`` distinct entries uniformly.
"""

from __future__ import annotations

import random
from typing import Any, Dict, List, Optional

import torch


class ReplayBuffer:
    def __init__(self, max_size: int = 10000) -> None:
        if max_size <= 0:
            raise ValueError(f"max_size must be positive, got {max_size}")
        self.max_size = max_size
        self._buffer: List[Dict[str, Any]] = []
        self._write_idx = 0

    @property
    def size(self) -> int:
        return len(self._buffer)

    def is_ready(self, min_size: int = 100) -> bool:
        return self.size >= min_size

    def add(self, input_ids: torch.Tensor, scores: Dict[str, torch.Tensor],
            metadata: Optional[Dict[str, Any]] = None) -> None:
        entry = {"input_ids": input_ids.detach().cpu(),
                 "scores": {k: v.detach().cpu() for k, v in scores.items()},
                 "metadata": metadata or {}}
        if self.size < self.max_size:
            self._buffer.append(entry)
        else:
            self._buffer[self._write_idx] = entry
        self._write_idx = (self._write_idx + 1) % self.max_size

    def add_batch(self, input_ids: torch.Tensor, scores: Dict[str, torch.Tensor],
                  metadata: Optional[Dict[str, Any]] = None) -> None:
        """Add each row of a (B, S) batch; one device→host copy for the whole batch."""
        ids = input_ids.detach().cpu()
        host = {k: v.detach().cpu() for k, v in scores.items()}
        for i in range(ids.size(0)):
            self.add(ids[i], {k: v[i] for k, v in host.items()}, metadata)

    def sample(self, batch_size: int) -> List[Dict[str, Any]]:
        if self.size == 0:
            return []
        return [self._buffer[i] for i in random.sample(range(self.size), min(batch_size, self.size))]

    def clear(self) -> None:
        self._buffer.clear()
        self._write_idx = 0

    def __len__(self) -> int:
        return self.size

    def __repr__(self) -> str:
        return f"ReplayBuffer(size={self.size}, max_size={self.max_size}, ready={self.is_ready()})"
