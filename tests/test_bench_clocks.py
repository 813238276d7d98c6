"""bench.py's clock sampler on a fake NVML (CPU): samples inside the marked timed window
are the ones reported, throttle-reason bits map to the contract's names, and without NVML
the sampler falls back without raising."""
import sys
import time
import types

import pytest


def _fake_nvml(clock_mhz, reasons_bits):
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    m.nvmlClocksEventReasonHwSlowdown = 0x8
    m.nvmlClocksEventReasonHwThermalSlowdown = 0x40
    m.nvmlClocksEventReasonSwThermalSlowdown = 0x20
    m.nvmlClocksEventReasonSwPowerCap = 0x4
    state = {"clock": clock_mhz, "bits": reasons_bits}
    m.nvmlInit = lambda: None
    m.nvmlShutdown = lambda: None
    m.nvmlDeviceGetHandleByIndex = lambda i: object()
    m.nvmlDeviceGetMaxClockInfo = lambda h, c: 1965
    m.nvmlDeviceGetClockInfo = lambda h, c: state["clock"]
    m.nvmlDeviceGetCurrentClocksEventReasons = lambda h: state["bits"]
    return m, state


@pytest.fixture
def bench_mod(monkeypatch):
    import importlib
    import bench
    return importlib.reload(bench)


def test_window_samples_and_reasons(bench_mod, monkeypatch):
    fake, state = _fake_nvml(1400, 0x0)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench_mod.ClockSampler(0) as clk:
        time.sleep(0.05)
        state["clock"], state["bits"] = 1965, 0x4          # under load: power cap only
        h0 = time.perf_counter()
        time.sleep(0.05)
        clk.window(h0, time.perf_counter())
        state["clock"], state["bits"] = 1000, 0x40         # after the window: ignored
        time.sleep(0.05)
    s = clk.summary()
    assert s["source"].startswith("nvml, inside")
    assert s["samples"] >= 3
    assert s["sm_mhz"] == 1965 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]


def test_without_nvml_falls_back(bench_mod, monkeypatch):
    broken = types.ModuleType("pynvml")

    def fail():
        raise RuntimeError("no NVML")
    broken.nvmlInit = fail
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    with bench_mod.ClockSampler(0) as clk:
        clk.window(time.perf_counter(), time.perf_counter())
    s = clk.summary()                                       # nvidia-smi absent here too
    assert "sm_mhz" in s and "reasons" in s
