"""Ring buffer of high-reward reasoning traces (``olympus/data/flywheel_buffer.py:17-194``).

Traces below ``reward_threshold`` are rejected; the oldest are evicted at
``max_size``.  Sampling is uniform without replacement, or with replacement
proportional to reward when ``priority_sampling``.
"""

from __future__ import annotations

import logging
import random
import time
from collections import deque
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional

logger = logging.getLogger(__name__)


@dataclass
class TraceEntry:
    context: str
    trace: str
    reward: float
    metadata: Dict[str, Any] = field(default_factory=dict)
    timestamp: float = 0.0


class FlywheelBuffer:
    def __init__(self, max_size: int = 100_000, reward_threshold: float = 0.1, priority_sampling: bool = False) -> None:
        self.max_size = max_size
        self.reward_threshold = reward_threshold
        self.priority_sampling = priority_sampling
        self._buffer: deque = deque(maxlen=max_size)
        self._total_added = 0
        self._total_rejected = 0

    def add(self, context: str, trace: str, reward: float, metadata: Optional[Dict[str, Any]] = None) -> bool:
        if reward < self.reward_threshold:
            self._total_rejected += 1
            return False
        self._buffer.append(TraceEntry(context, trace, float(reward), dict(metadata or {}), time.time()))
        self._total_added += 1
        return True

    def sample(self, batch_size: int) -> List[Dict[str, Any]]:
        if not self._buffer:
            return []
        n = min(batch_size, len(self._buffer))
        pool = list(self._buffer)
        if self.priority_sampling:
            picked = random.choices(pool, weights=[max(e.reward, 1e-8) for e in pool], k=n)
        else:
            picked = random.sample(pool, n)
        return [{"context": e.context, "trace": e.trace, "reward": e.reward, "metadata": e.metadata} for e in picked]

    @property
    def size(self) -> int:
        return len(self._buffer)

    def __len__(self) -> int:
        return len(self._buffer)

    def stats(self) -> Dict[str, Any]:
        r = [e.reward for e in self._buffer]
        return {
            "size": len(r), "max_size": self.max_size, "total_added": self._total_added,
            "total_rejected": self._total_rejected, "avg_reward": sum(r) / len(r) if r else 0.0,
            "min_reward": min(r) if r else 0.0, "max_reward": max(r) if r else 0.0,
        }

    def clear(self) -> None:
        self._buffer.clear()

    def state_dict(self) -> Dict[str, Any]:
        return {"entries": [asdict(e) for e in self._buffer], "total_added": self._total_added,
                "total_rejected": self._total_rejected, "max_size": self.max_size,
                "reward_threshold": self.reward_threshold, "priority_sampling": self.priority_sampling}

    def load_state_dict(self, state: Dict[str, Any]) -> None:
        self.max_size = state.get("max_size", self.max_size)
        self.reward_threshold = state.get("reward_threshold", self.reward_threshold)
        self.priority_sampling = state.get("priority_sampling", self.priority_sampling)
        self._buffer = deque((TraceEntry(**e) for e in state.get("entries", [])), maxlen=self.max_size)
        self._total_added = state.get("total_added", 0)
        self._total_rejected = state.get("total_rejected", 0)
