"""Host-side pieces of bench.py that need no GPU: the SM-clock sampler that
backs the line's "clocks" record (through a fake NVML module) and its
fallbacks."""

import sys
import time
import types

import pytest


class _FakeNvml(types.ModuleType):
    NVML_CLOCK_SM = 1

    def __init__(self, clocks, reasons):
        super().__init__("pynvml")
        self._clocks = list(clocks)
        self._reasons = reasons
        self.calls = 0

    def nvmlInit(self):
        pass

    def nvmlDeviceGetHandleByUUID(self, uuid):
        raise RuntimeError("no uuid on this host")

    def nvmlDeviceGetHandleByIndex(self, index):
        return ("gpu", index)

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        assert kind == self.NVML_CLOCK_SM
        return 1965

    def nvmlDeviceGetClockInfo(self, h, kind):
        self.calls += 1
        return self._clocks[min(self.calls - 1, len(self._clocks) - 1)]

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return self._reasons


@pytest.fixture
def bench_mod():
    import importlib.util
    from pathlib import Path

    spec = importlib.util.spec_from_file_location("bench_under_test", Path(__file__).resolve().parents[1] / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_sampler_nvml_reasons_and_median(bench_mod, monkeypatch):
    fake = _FakeNvml([1965, 1950, 1965, 1900, 1965], 0x4 | 0x8)  # sw_power_cap | hw_slowdown
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    clk = bench_mod.ClockSampler(0)
    assert clk.source == "nvml"
    with clk:
        clk.mark()
        time.sleep(0.05)
        clk.sample_now()
    s = clk.summary()
    assert s["source"] == "nvml" and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert s["samples"] >= 1 and 1900.0 <= s["sm_mhz"] <= 1965.0


def test_clock_sampler_short_region_keeps_last_sample(bench_mod, monkeypatch):
    """A timed region shorter than one sampling period still reports the
    sample taken just before it opened."""
    fake = _FakeNvml([1965], 0)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    clk = bench_mod.ClockSampler(0)
    clk._run = lambda: clk.samples.append(clk._sample_nvml())  # one sample, then stop
    with clk:
        clk.mark()
    s = clk.summary()
    assert s["samples"] == 1 and s["sm_mhz"] == 1965.0 and s["reasons"] == []


def test_clock_sampler_without_nvml_falls_back(bench_mod, monkeypatch):
    broken = types.ModuleType("pynvml")  # no nvmlInit: NVML unusable
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    clk = bench_mod.ClockSampler(0)
    assert clk.source == "nvidia-smi"
    clk.sample_now()  # a no-op without NVML
    assert clk.summary()["reasons"] == ["unsampled"]
