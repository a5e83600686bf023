"""decode_opt_b200.clocks.ClockSampler against a fake NVML (no GPU): the clock
record bench.py attaches to its JSON line.  The fake exposes getters only, so
the sampler reading anything else -- let alone setting a clock -- fails the
test."""

import sys
import time
import types

import pytest

from decode_opt_b200 import clocks


def _fake_nvml(mhz_seq, reasons_seq, max_mhz=1965):
    state = {"i": 0}
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    m.nvmlInit = lambda: None
    m.nvmlDeviceGetHandleByIndex = lambda i: ("handle", i)
    m.nvmlDeviceGetMaxClockInfo = lambda h, kind: max_mhz

    def clock(h, kind):
        i = min(state["i"], len(mhz_seq) - 1)
        return mhz_seq[i]

    def reasons(h):
        i = min(state["i"], len(reasons_seq) - 1)
        state["i"] += 1
        return reasons_seq[i]

    m.nvmlDeviceGetClockInfo = clock
    m.nvmlDeviceGetCurrentClocksEventReasons = reasons
    return m


@pytest.fixture
def fake(monkeypatch):
    def install(mhz, reasons):
        monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(mhz, reasons))
        return clocks.ClockSampler(0, period_s=0.001)
    return install


def test_reason_names_skip_idle_and_decode_bits(fake):
    cs = fake([1965], [0])
    assert cs.reason_names(0x1 | 0x4) == ["sw_power_cap"]
    assert cs.reason_names(0x8 | 0x40 | 0x20) == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]
    assert cs.reason_names(0) == []


def test_summary_uses_marked_interval(fake):
    cs = fake([1965], [0])
    assert cs.available and cs.max_mhz == 1965
    cs.samples = [(0.0, 1000, 0x0), (1.0, 1965, 0x0), (2.0, 1600, 0x4), (3.0, 1500, 0x4), (9.0, 500, 0x8)]
    cs._marks = [0.5, 3.5]
    s = cs.summary()
    assert s["sm_mhz"] == 1600 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]          # the hw_slowdown sample lies outside the marks
    assert cs.median_between(0.5, 3.5) == 1600
    assert cs.median_between(5.0, 6.0) == 1500        # nearest sample when none falls inside


def test_thread_collects_samples(fake):
    cs = fake([1965, 1965, 1700, 1600], [0, 0, 0x4, 0x4])
    cs.start()
    cs.mark()
    time.sleep(0.05)
    cs.mark()
    cs.stop()
    assert len(cs.samples) >= 2
    s = cs.summary()
    assert s["sm_max_mhz"] == 1965 and 1600 <= s["sm_mhz"] <= 1965


def test_without_nvml_reports_no_clocks(monkeypatch):
    broken = types.ModuleType("pynvml")

    def fail():
        raise RuntimeError("no NVML")
    broken.nvmlInit = fail
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    cs = clocks.ClockSampler(0)
    assert not cs.available
    assert cs.read_now() == (None, 0)
    cs.start()
    cs.stop()
    assert cs.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
