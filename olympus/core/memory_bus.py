"""Scoped key/value tensor store shared between models.

Three scopes, as in ``olympus/core/memory_bus.py:22-161`` of the reference:

``step``       cleared by :meth:`MemoryBus.step` at the end of every training step;
``episode``    cleared on demand with :meth:`MemoryBus.clear_episode`;
``permanent``  never cleared automatically and saved in checkpoints.

Values are stored as detached copies and handed out as copies, so callers can
never alias the bus contents.  All access is serialised by one lock.
"""

from __future__ import annotations

import threading
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

SCOPES = ("step", "episode", "permanent")
_VALID_SCOPES = set(SCOPES)


class MemoryBus:
    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._stores: Dict[str, Dict[str, torch.Tensor]] = {s: {} for s in SCOPES}

    @staticmethod
    def _validate_scope(scope: str) -> None:
        if scope not in _VALID_SCOPES:
            raise ValueError(f"Invalid scope '{scope}'. Must be one of {sorted(_VALID_SCOPES)}.")

    def write(self, key: str, value: torch.Tensor, scope: str = "step") -> None:
        self._validate_scope(scope)
        copy = value.detach().clone()
        with self._lock:
            self._stores[scope][key] = copy

    def read(self, key: str, scope: str = "step") -> Optional[torch.Tensor]:
        self._validate_scope(scope)
        with self._lock:
            val = self._stores[scope].get(key)
            return None if val is None else val.clone()

    def query(self, query_vector: torch.Tensor, scope: str = "step", top_k: int = 5) -> List[Tuple[str, torch.Tensor, float]]:
        """Rank every entry of ``scope`` by cosine similarity to ``query_vector``.

        Entries and the query are flattened; when lengths differ the shorter one
        is zero-padded, so any two tensors can be compared.
        """
        self._validate_scope(scope)
        q = query_vector.detach().reshape(-1).float()
        with self._lock:
            items = [(k, v) for k, v in self._stores[scope].items()]
        scored: List[Tuple[str, torch.Tensor, float]] = []
        for key, tensor in items:
            t = tensor.reshape(-1).float().to(q.device)
            n = max(t.numel(), q.numel())
            a = F.pad(q, (0, n - q.numel()))
            b = F.pad(t, (0, n - t.numel()))
            sim = float(F.cosine_similarity(a[None], b[None]).item())
            scored.append((key, tensor.clone(), sim))
        scored.sort(key=lambda r: r[2], reverse=True)
        return scored[:top_k]

    def list_keys(self, scope: str = "step") -> List[str]:
        self._validate_scope(scope)
        with self._lock:
            return list(self._stores[scope])

    def step(self) -> None:
        with self._lock:
            self._stores["step"].clear()

    def clear_episode(self) -> None:
        with self._lock:
            self._stores["episode"].clear()

    def clear_all(self) -> None:
        with self._lock:
            for store in self._stores.values():
                store.clear()

    def state_dict(self) -> Dict[str, Dict[str, torch.Tensor]]:
        """Snapshot of the ``permanent`` and ``episode`` scopes (CPU copies)."""
        with self._lock:
            return {
                scope: {k: v.detach().cpu().clone() for k, v in self._stores[scope].items()}
                for scope in ("permanent", "episode")
            }

    def load_state_dict(self, state: Dict[str, Dict[str, torch.Tensor]]) -> None:
        with self._lock:
            for scope in ("permanent", "episode"):
                if scope in state:
                    self._stores[scope] = {k: v.clone() for k, v in state[scope].items()}

    def __repr__(self) -> str:
        with self._lock:
            counts = ", ".join(f"{s}={len(self._stores[s])}" for s in SCOPES)
        return f"MemoryBus({counts})"
