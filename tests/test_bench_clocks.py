"""bench.py's clock sampler against a fake NVML module (CPU only; nothing touches a GPU)."""
import os
import sys
import time
import types

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


def _fake_nvml(clocks, reasons):
    state = {"i": 0, "inits": 0, "shutdowns": 0}
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1

    def nvmlInit():
        state["inits"] += 1

    def nvmlShutdown():
        state["shutdowns"] += 1

    def handle(*a):
        return "h"

    def clock(h, kind):
        assert kind == 1
        v = clocks[min(state["i"], len(clocks) - 1)]
        return v

    def max_clock(h, kind):
        return 1965

    def ev(h):
        r = reasons[min(state["i"], len(reasons) - 1)]
        state["i"] += 1
        return r

    m.nvmlInit, m.nvmlShutdown = nvmlInit, nvmlShutdown
    m.nvmlDeviceGetHandleByIndex = handle
    m.nvmlDeviceGetHandleByPciBusId = handle
    m.nvmlDeviceGetClockInfo, m.nvmlDeviceGetMaxClockInfo = clock, max_clock
    m.nvmlDeviceGetCurrentClocksEventReasons = ev
    return m, state


def test_nvml_sampler_reports_median_and_reasons(monkeypatch):
    fake, state = _fake_nvml([1965, 1965, 1800, 1965], [0, 0x4, 0x4 | 0x40, 0])
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    c = bench.ClockSampler(0, period_s=0.002)
    with c:
        time.sleep(0.05)
    s = c.summary()
    assert s["source"].startswith("nvml")
    assert s["samples"] >= 4
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
    assert state["inits"] == 1 and state["shutdowns"] == 1


def test_sampler_takes_a_sample_before_the_region():
    """The first NVML sample exists by the time the with-block starts."""
    fake, _ = _fake_nvml([1965], [0])
    sys.modules["pynvml"], old = fake, sys.modules.get("pynvml")
    try:
        c = bench.ClockSampler(0, period_s=10.0)
        with c:
            assert len(c.samples) == 1
        assert c.summary()["samples"] == 1
    finally:
        if old is None:
            sys.modules.pop("pynvml", None)
        else:
            sys.modules["pynvml"] = old


def test_sampler_without_nvml_or_gpu_reports_no_samples(monkeypatch):
    broken = types.ModuleType("pynvml")

    def fail():
        raise RuntimeError("no NVML")

    broken.nvmlInit = fail
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    monkeypatch.setattr(bench.subprocess, "Popen", lambda *a, **k: (_ for _ in ()).throw(FileNotFoundError()))
    c = bench.ClockSampler(0)
    with c:
        pass
    assert c.summary()["samples"] == 0
