"""Running metric tracker (``olympus/utils/metrics.py:10-133``).

Windowed and all-time averages, last/min/max/count per metric; ``dump``
flattens them as ``{name}/avg``, ``{name}/global_avg``, ``{name}/last``,
``{name}/min``, ``{name}/max``, ``{name}/count``.  Values may be 0-d device
tensors (they are converted when read, so updates never synchronise).
"""

from __future__ import annotations

from collections import defaultdict, deque
from typing import Any, Deque, Dict, Optional


def _f(v: Any) -> float:
    return float(v)


class MetricsAggregator:
    def __init__(self, window_size: int = 100) -> None:
        self.window_size = window_size
        self.reset()

    def reset(self) -> None:
        self._values: Dict[str, Deque[Any]] = defaultdict(lambda: deque(maxlen=self.window_size))
        self._last: Dict[str, Any] = {}
        self._sums: Dict[str, float] = defaultdict(float)
        self._counts: Dict[str, int] = defaultdict(int)
        self._min: Dict[str, float] = {}
        self._max: Dict[str, float] = {}
        self._pending: Dict[str, list] = defaultdict(list)

    def update(self, metrics: Dict[str, Any]) -> None:
        for k, v in metrics.items():
            self._last[k] = v
            self._values[k].append(v)
            self._counts[k] += 1
            self._pending[k].append(v)

    def _settle(self, k: str) -> None:
        for v in self._pending.pop(k, []):
            x = _f(v)
            self._sums[k] += x
            self._min[k] = x if k not in self._min else min(self._min[k], x)
            self._max[k] = x if k not in self._max else max(self._max[k], x)

    def get_last(self, key: str, default: float = 0.0) -> float:
        return _f(self._last[key]) if key in self._last else default

    def get_average(self, key: str, default: float = 0.0) -> float:
        vals = self._values.get(key)
        return sum(_f(v) for v in vals) / len(vals) if vals else default

    def get_global_average(self, key: str, default: float = 0.0) -> float:
        self._settle(key)
        n = self._counts.get(key, 0)
        return self._sums[key] / n if n else default

    def get_min(self, key: str) -> Optional[float]:
        self._settle(key)
        return self._min.get(key)

    def get_max(self, key: str) -> Optional[float]:
        self._settle(key)
        return self._max.get(key)

    def get_count(self, key: str) -> int:
        return self._counts.get(key, 0)

    def to_dict(self) -> Dict[str, float]:
        return {k: _f(v) for k, v in self._last.items()}

    def averages(self) -> Dict[str, float]:
        return {k: self.get_average(k) for k in self._values}

    def dump(self, reset: bool = False) -> Dict[str, float]:
        out: Dict[str, float] = {}
        for k in list(self._counts):
            out[f"{k}/avg"] = self.get_average(k)
            out[f"{k}/global_avg"] = self.get_global_average(k)
            if k in self._last:
                out[f"{k}/last"] = _f(self._last[k])
            if k in self._min:
                out[f"{k}/min"] = self._min[k]
            if k in self._max:
                out[f"{k}/max"] = self._max[k]
            out[f"{k}/count"] = float(self._counts[k])
        if reset:
            self.reset()
        return out
