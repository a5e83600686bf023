"""SM clock and throttle-reason sampling through NVML (read-only).

The benchmarks record the SM clock seen while they time (the reference writes
`nvidia-smi --query-gpu=clocks.sm` into every CSV row,
bench/bench_decode.cu:669-687).  Nothing here changes a GPU setting.
"""

from __future__ import annotations

import statistics
import threading
import time


class ClockSampler:
    """Samples the SM clock and the clock-event reasons every ~20 ms on a
    background thread; `summary()` and `median_between()` read the samples."""

    REASONS = {  # nvmlClocksEventReason* bits
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.02):
        self.samples = []
        self.max_mhz = None
        self.period_s = period_s
        self._stop = threading.Event()
        self._thread = None
        self._marks = []
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - NVML missing: report no clocks
            self._nvml = None

    @property
    def available(self) -> bool:
        return self._nvml is not None

    def read_now(self):
        """(SM MHz, reason bits) read once, or (None, 0)."""
        if self._nvml is None:
            return None, 0
        nv = self._nvml
        try:
            return nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM), \
                nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:  # noqa: BLE001
            return None, 0

    def _run(self):
        while not self._stop.is_set():
            mhz, reasons = self.read_now()
            if mhz is not None:
                self.samples.append((time.perf_counter(), mhz, reasons))
            self._stop.wait(self.period_s)

    def start(self):
        if self._nvml is not None and self._thread is None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def mark(self):
        self._marks.append(time.perf_counter())

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=1.0)

    def reason_names(self, bits: int):
        return sorted(name for bit, name in self.REASONS.items() if bits & bit and name != "gpu_idle")

    def median_between(self, t0: float, t1: float):
        """Median SM MHz of the samples taken in [t0, t1] (perf_counter
        seconds); the sample nearest the interval when none fell inside; None
        without NVML."""
        inside = [s[1] for s in self.samples if t0 <= s[0] <= t1]
        if inside:
            return statistics.median(inside)
        if self.samples:
            mid = 0.5 * (t0 + t1)
            return min(self.samples, key=lambda s: abs(s[0] - mid))[1]
        return self.read_now()[0]

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        lo, hi = (self._marks[0], self._marks[-1]) if len(self._marks) >= 2 else (-1e30, 1e30)
        inside = [s for s in self.samples if lo <= s[0] <= hi] or self.samples
        mhz = statistics.median(s[1] for s in inside)
        bits = 0
        for s in inside:
            bits |= s[2]
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": self.reason_names(bits),
                "samples": len(inside)}
