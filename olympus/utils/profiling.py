"""Memory and timing instrumentation (``olympus/utils/profiling.py:13-130``) plus
device-side phase timing.

* ``get_gpu_memory_stats`` / ``reset_peak_memory`` / ``count_parameters`` /
  ``MemoryTracker`` -- as in the reference.
* :class:`DeviceTimer` -- CUDA-event timing of named phases on the launching
  stream (no host synchronisation until ``summary()``), with an NVTX range per
  phase for external profilers, and a max-over-ranks reduction for
  multi-GPU runs.
"""

from __future__ import annotations

import contextlib
import logging
from collections import defaultdict
from typing import Any, Dict, Iterator, List, Optional, Tuple

import torch
import torch.nn as nn

logger = logging.getLogger(__name__)


def get_gpu_memory_stats(device: Optional[int] = None) -> Dict[str, float]:
    if not torch.cuda.is_available():
        return {}
    dev = torch.cuda.current_device() if device is None else device
    gb = 1024 ** 3
    free, total = torch.cuda.mem_get_info(dev)
    return {
        "allocated_gb": torch.cuda.memory_allocated(dev) / gb,
        "reserved_gb": torch.cuda.memory_reserved(dev) / gb,
        "max_allocated_gb": torch.cuda.max_memory_allocated(dev) / gb,
        "max_reserved_gb": torch.cuda.max_memory_reserved(dev) / gb,
        "free_gb": free / gb,
        "total_gb": total / gb,
    }


def reset_peak_memory(device: Optional[int] = None) -> None:
    if torch.cuda.is_available():
        torch.cuda.reset_peak_memory_stats(device)


def count_parameters(model: nn.Module, trainable_only: bool = False) -> Dict[str, int]:
    total = sum(p.numel() for p in model.parameters())
    trainable = sum(p.numel() for p in model.parameters() if p.requires_grad)
    return {"total": total, "trainable": trainable, "frozen": total - trainable} if not trainable_only else {"trainable": trainable}


class MemoryTracker:
    """``with MemoryTracker("fwd") as mt: ...`` -> ``mt.delta_gb`` / ``mt.peak_gb``."""

    def __init__(self, label: str = "", device: Optional[int] = None, log: bool = True) -> None:
        self.label = label
        self.device = device
        self.log = log
        self.delta_gb = 0.0
        self.peak_gb = 0.0

    def __enter__(self) -> "MemoryTracker":
        if torch.cuda.is_available():
            torch.cuda.synchronize(self.device)
            torch.cuda.reset_peak_memory_stats(self.device)
            self._start = torch.cuda.memory_allocated(self.device)
        return self

    def __exit__(self, *exc: Any) -> None:
        if torch.cuda.is_available():
            torch.cuda.synchronize(self.device)
            gb = 1024 ** 3
            self.delta_gb = (torch.cuda.memory_allocated(self.device) - self._start) / gb
            self.peak_gb = torch.cuda.max_memory_allocated(self.device) / gb
            if self.log:
                logger.info("[%s] memory delta %.3f GB, peak %.3f GB", self.label, self.delta_gb, self.peak_gb)


class DeviceTimer:
    """Accumulates CUDA-event durations per phase name."""

    def __init__(self, enabled: bool = True) -> None:
        self.enabled = enabled and torch.cuda.is_available()
        self._events: Dict[str, List[Tuple[torch.cuda.Event, torch.cuda.Event]]] = defaultdict(list)

    @contextlib.contextmanager
    def phase(self, name: str) -> Iterator[None]:
        if not self.enabled:
            yield
            return
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(name)
        a.record()
        try:
            yield
        finally:
            b.record()
            torch.cuda.nvtx.range_pop()
            self._events[name].append((a, b))

    def summary(self, reduce_max_over_ranks: bool = False) -> Dict[str, float]:
        """Milliseconds per phase (synchronises)."""
        if not self.enabled:
            return {}
        torch.cuda.synchronize()
        out = {k: sum(a.elapsed_time(b) for a, b in v) for k, v in self._events.items()}
        if reduce_max_over_ranks:
            import torch.distributed as dist

            if dist.is_initialized() and out:
                keys = sorted(out)
                t = torch.tensor([out[k] for k in keys], device="cuda", dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                out = dict(zip(keys, t.tolist()))
        return out

    def reset(self) -> None:
        self._events.clear()
