"""GPU clock / throttle-reason sampling through NVML (read-only).

Used by bench.py to record the SM clock and active clock-event reasons
while the timed region runs.  Nothing here changes a GPU setting.
"""

from __future__ import annotations

import statistics
import threading
import time
from typing import Dict, List, Optional

# NVML clocks-event-reason bits (nvml.h, nvmlClocksEventReason*)
_REASONS = {
    0x1: "gpu_idle",
    0x2: "applications_clocks_setting",
    0x4: "sw_power_cap",
    0x8: "hw_slowdown",
    0x10: "sync_boost",
    0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


def decode_reasons(mask: int) -> List[str]:
    return [name for bit, name in _REASONS.items() if mask & bit]


class ClockSampler:
    """Background thread sampling SM clock and clock-event reasons every `period_s`."""

    def __init__(self, device_index: int = 0, period_s: float = 0.005) -> None:
        self.period_s = period_s
        self.samples: List[Dict] = []
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._h = None
        self.max_mhz: Optional[int] = None
        self.error: Optional[str] = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = int(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception as e:  # pragma: no cover - depends on the host
            self.error = f"nvml unavailable: {e}"

    def _reasons(self) -> int:
        nv = self._nv
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
            nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
        return int(fn(self._h))

    def _run(self) -> None:
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append({
                    "t": time.perf_counter(),
                    "sm_mhz": int(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)),
                    "reasons": self._reasons(),
                })
            except Exception as e:  # pragma: no cover
                self.error = str(e)
                return
            self._stop.wait(self.period_s)

    def start(self) -> "ClockSampler":
        if self._h is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2.0)

    def summary(self, t0: Optional[float] = None, t1: Optional[float] = None) -> Dict:
        """Median SM clock and union of reasons over samples in [t0, t1] (all if None)."""
        s = [x for x in self.samples if (t0 is None or x["t"] >= t0) and (t1 is None or x["t"] <= t1)]
        if not s:
            s = self.samples
        mask = 0
        for x in s:
            mask |= x["reasons"]
        out = {
            "sm_mhz": statistics.median([x["sm_mhz"] for x in s]) if s else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(set(decode_reasons(mask)) - {"gpu_idle"}),
            "samples": len(s),
        }
        if self.error:
            out["error"] = self.error
        return out
