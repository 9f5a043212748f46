"""CPU: bench.py's clock sampler against a fake NVML (no GPU; nothing is changed on a GPU).

The sampler reads the SM clock, the maximum SM clock and the clock-event reason mask
from NVML every 10 ms while the timed steps run; the summary reports the median clock
and every reason seen, named as the bench line's ``clocks.reasons`` expects."""
import sys
import time
import types
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import bench  # noqa: E402


def _fake_nvml(clocks, mask):
    fake = types.ModuleType("pynvml")
    fake.NVML_CLOCK_SM = 1
    fake.nvmlInit = lambda: None
    fake.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    fake.nvmlDeviceGetMaxClockInfo = lambda h, c: 1965
    it = iter(clocks)
    fake.nvmlDeviceGetClockInfo = lambda h, c: next(it, clocks[-1])
    fake.nvmlDeviceGetCurrentClocksEventReasons = lambda h: mask
    return fake


def test_sampler_reports_median_clock_and_named_reasons(monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml([1800, 1900, 1965, 1900, 1850], 0x4 | 0x20))
    with bench.ClockSampler(0) as c:
        time.sleep(0.15)
    s = c.summary()
    assert s["samples"] >= 5
    assert s["sm_max_mhz"] == 1965.0
    assert 1800.0 <= s["sm_mhz"] <= 1965.0
    assert s["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]


def test_sampler_with_no_reasons_active(monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml([1965], 0x0))
    with bench.ClockSampler(0) as c:
        time.sleep(0.05)
    s = c.summary()
    assert s["reasons"] == [] and s["sm_mhz"] == 1965.0
