"""Read-only sampling of GPU clocks and clock-event (throttle) reasons.

Runs NVML queries on a background thread during a timed region. Nothing here
changes any GPU setting.
"""
from __future__ import annotations

import statistics
import threading
import time

_REASONS = {
    0x0000000000000001: "gpu_idle",
    0x0000000000000002: "applications_clocks_setting",
    0x0000000000000004: "sw_power_cap",
    0x0000000000000008: "hw_slowdown",
    0x0000000000000010: "sync_boost",
    0x0000000000000020: "sw_thermal_slowdown",
    0x0000000000000040: "hw_thermal_slowdown",
    0x0000000000000080: "hw_power_brake_slowdown",
    0x0000000000000100: "display_clock_setting",
}


def decode_reasons(mask: int) -> list[str]:
    return [name for bit, name in _REASONS.items() if mask & bit]


class ClockSampler:
    """Samples SM clock, power and event reasons of `devices` every `period_s`."""

    def __init__(self, devices, period_s: float = 0.02):
        self.devices = list(devices)
        self.period_s = period_s
        self.samples = []  # (t, dev, sm_mhz, power_w, reasons_mask)
        self._stop = threading.Event()
        self._th = None
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = [pynvml.nvmlDeviceGetHandleByIndex(d) for d in self.devices]
            self.max_mhz = max(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM) for h in self._h)
            self.ok = True
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        getr = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
            nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
        while not self._stop.is_set():
            t = time.time()
            for d, h in zip(self.devices, self._h):
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                    rs = getr(h)
                    self.samples.append((t, d, mhz, pw, rs))
                except Exception:
                    pass
            self._stop.wait(self.period_s)

    def start(self):
        if self.ok:
            self._th = threading.Thread(target=self._run, daemon=True)
            self._th.start()
        return self

    def stop(self):
        if self._th is not None:
            self._stop.set()
            self._th.join()
        return self

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        busy = [s for s in self.samples if not (s[4] & 0x1)] or self.samples
        mask = 0
        for s in busy:
            mask |= s[4]
        return {
            "sm_mhz": statistics.median(s[2] for s in busy),
            "sm_max_mhz": self.max_mhz,
            "power_w_max": max(s[3] for s in self.samples),
            "reasons": [r for r in decode_reasons(mask) if r != "gpu_idle"],
            "samples": len(self.samples),
        }
