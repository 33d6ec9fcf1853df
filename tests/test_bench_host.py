"""Host-side pieces of bench.py that need no GPU: the clock sampler against a
stand-in NVML module (read-only queries; it sets nothing on any GPU)."""
import sys
import time
import types

import bench


def test_clock_sampler_reports_median_max_and_reasons(monkeypatch):
    clocks = iter([1900.0, 1905.0, 1910.0] + [1905.0] * 10000)
    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=0,
        nvmlInit=lambda: None,
        nvmlDeviceGetHandleByIndex=lambda i: ("gpu", i),
        nvmlDeviceGetMaxClockInfo=lambda h, c: 1965,
        nvmlDeviceGetClockInfo=lambda h, c: next(clocks),
        # sw_power_cap | hw_slowdown, plus a bit the sampler does not name
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x4 | 0x8 | 0x1,
    )
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.Clocks(0, period_s=0.001) as c:
        time.sleep(0.02)
    s = c.summary()
    assert s["sm_max_mhz"] == 1965.0
    assert s["samples"] >= 1 and 1900.0 <= s["sm_mhz"] <= 1910.0
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_clock_sampler_without_nvml(monkeypatch):
    """No NVML: the bench still runs and reports no clock samples."""
    monkeypatch.setitem(sys.modules, "pynvml", None)  # import raises ImportError
    with bench.Clocks(0) as c:
        pass
    s = c.summary()
    assert s["samples"] == 0 and s["sm_mhz"] is None and s["reasons"] == []
