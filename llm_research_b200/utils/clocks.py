"""Read-only GPU clock / throttle sampling through NVML (nothing is ever set)."""

from __future__ import annotations

import statistics
import threading
import time
from typing import Dict, List, Optional

_REASONS = {
    "gpu_idle": 0x1,
    "applications_clocks_setting": 0x2,
    "sw_power_cap": 0x4,
    "hw_slowdown": 0x8,
    "sync_boost": 0x10,
    "sw_thermal_slowdown": 0x20,
    "hw_thermal_slowdown": 0x40,
    "hw_power_brake_slowdown": 0x80,
    "display_clock_setting": 0x100,
}


class ClockSampler:
    """Samples SM clock, power and active throttle reasons every ``period_s``."""

    def __init__(self, device_index: int = 0, period_s: float = 0.2) -> None:
        self.period = period_s
        self.samples: List[Dict[str, float]] = []
        self.reasons: set = set()
        self.max_mhz: Optional[float] = None
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._ok = False
        try:
            import pynvml  # nvidia_ml_py

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
            self._ok = True
        except Exception:
            self._ok = False

    def _run(self) -> None:
        nv = self._nvml
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                util = nv.nvmlDeviceGetUtilizationRates(self._h).gpu
                self.samples.append({"sm_mhz": float(sm), "power_w": pw, "util": float(util)})
                for name, bit in _REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self) -> "ClockSampler":
        if self._ok:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2.0)

    def summary(self) -> Dict[str, object]:
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        loaded = [s["sm_mhz"] for s in self.samples if s["util"] > 50] or [s["sm_mhz"] for s in self.samples]
        return {
            "sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
            "power_w_max": max((s["power_w"] for s in self.samples), default=None),
        }
