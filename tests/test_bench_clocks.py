"""bench.py's clock sampler against a fake NVML (no GPU): it keeps only samples taken after
begin(), decodes the clocks-event reason bits, and reports median / max clocks and power."""
import os
import sys
import time
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _fake_nvml(state):
    nv = types.ModuleType("pynvml")
    nv.NVML_CLOCK_SM = 1
    nv.nvmlInit = lambda: state.setdefault("init", True)
    nv.nvmlShutdown = lambda: state.setdefault("shutdown", True)

    def by_bus(bus):
        raise RuntimeError("no bus ids in the fake")

    nv.nvmlDeviceGetHandleByPciBusId = by_bus
    nv.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    nv.nvmlDeviceGetClockInfo = lambda h, kind: state["sm"]
    nv.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965
    nv.nvmlDeviceGetPowerUsage = lambda h: state["mw"]
    nv.nvmlDeviceGetCurrentClocksEventReasons = lambda h: state["bits"]
    return nv


def test_clock_sampler_nvml_window_and_reasons(monkeypatch):
    import bench
    state = {"sm": 300, "mw": 90_000, "bits": 1}  # idle before the timed region
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(state))
    cs = bench.ClockSampler([0])
    cs.start()
    assert cs.nvml is not None
    time.sleep(0.1)
    assert cs.samples == [], "samples kept before begin()"
    state.update(sm=1600, mw=998_000, bits=4)  # power-capped under load
    cs.begin()
    time.sleep(0.15)
    out = cs.stop()
    assert state.get("shutdown")
    assert out["samples"] >= 3
    assert out["sm_mhz"] == 1600 and out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"]
    assert out["power_w_max"] == 998.0


def test_clock_sampler_decodes_every_reason_bit(monkeypatch):
    import bench
    state = {"sm": 1000, "mw": 500_000, "bits": 8 | 32 | 64}
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(state))
    cs = bench.ClockSampler([0])
    cs.start()
    cs.begin()
    time.sleep(0.06)
    out = cs.stop()
    assert out["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]
