"""bench.py's clock sampler against a fake NVML (CPU, no GPU): samples are
taken during a timed region even when it is shorter than NVML's start-up,
and throttle reasons are decoded from the clocks-event bits."""

from __future__ import annotations

import importlib.util
import sys
import time
import types
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def fake_nvml(init_seconds: float, reasons: int) -> types.ModuleType:
    nvml = types.ModuleType("pynvml")
    nvml.NVML_CLOCK_SM = 1
    nvml.nvmlInit = lambda: time.sleep(init_seconds)
    nvml.nvmlDeviceGetHandleByIndex = lambda index: ("gpu", index)
    nvml.nvmlDeviceGetMaxClockInfo = lambda handle, clock: 1965
    nvml.nvmlDeviceGetClockInfo = lambda handle, clock: 1950
    nvml.nvmlDeviceGetCurrentClocksEventReasons = lambda handle: reasons
    nvml.nvmlDeviceGetPowerUsage = lambda handle: 640_000
    return nvml


@pytest.fixture
def bench(monkeypatch):
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    return load_bench()


def test_short_region_after_slow_nvml_start_is_sampled(bench, monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", fake_nvml(0.3, 0))
    with bench.ClockSampler(0) as clocks:
        time.sleep(0.005)  # a region far shorter than NVML's start-up
    summary = clocks.summary()
    assert summary["samples"] >= 2 and summary["sm_mhz"] == 1950 and summary["sm_max_mhz"] == 1965
    assert summary["reasons"] == [] and summary["power_w_max"] == 640.0


def test_throttle_reasons_are_decoded(bench, monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", fake_nvml(0.0, 0x4 | 0x40))
    with bench.ClockSampler(0) as clocks:
        time.sleep(0.01)
    assert clocks.summary()["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]


def test_missing_nvml_is_reported_not_raised(bench, monkeypatch):
    broken = types.ModuleType("pynvml")

    def refuse():
        raise RuntimeError("no NVML here")

    broken.nvmlInit = refuse
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    with bench.ClockSampler(0) as clocks:
        pass
    summary = clocks.summary()
    assert summary["samples"] == 0 and "no NVML here" in summary["error"]
