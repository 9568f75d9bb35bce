"""bench.py host logic without a GPU: the NVML clock sampler that runs
during the timed region (median SM clock, max clock, clock-event reasons
seen), driven by a fake NVML module."""
import sys
import time
import types

import bench

SW_POWER_CAP, SW_THERMAL = 0x4, 0x20


def _fake_nvml(monkeypatch, samples, fail=False):
    """A stand-in pynvml whose SM clock and reasons cycle through `samples`."""
    nv = types.ModuleType("pynvml")
    nv.NVML_CLOCK_SM = 1
    state = {"i": 0}

    def init():
        if fail:
            raise RuntimeError("no NVML here")

    def clock(h, which):
        sm, _ = samples[state["i"] % len(samples)]
        return sm

    def reasons(h):
        _, bits = samples[state["i"] % len(samples)]
        state["i"] += 1
        return bits

    nv.nvmlInit = init
    nv.nvmlDeviceGetHandleByUUID = lambda u: "h"
    nv.nvmlDeviceGetHandleByIndex = lambda i: "h"
    nv.nvmlDeviceGetMaxClockInfo = lambda h, which: 1965
    nv.nvmlDeviceGetClockInfo = clock
    nv.nvmlDeviceGetPowerUsage = lambda h: 700500
    nv.nvmlDeviceGetCurrentClocksEventReasons = reasons
    monkeypatch.setitem(sys.modules, "pynvml", nv)


def test_clock_sampler_reports_median_and_reasons(monkeypatch):
    _fake_nvml(monkeypatch, [(1965, SW_POWER_CAP), (1800, SW_POWER_CAP)])
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.2)
    r = s.stop()
    assert r["samples"] >= 2  # one at each end at least, however short the region
    assert r["sm_max_mhz"] == 1965.0
    assert 1800.0 <= r["sm_mhz"] <= 1965.0
    assert r["power_w"] == 700.5
    assert r["reasons"] == ["sw_power_cap"]  # power cap is kept and noted


def test_clock_sampler_short_region_still_samples(monkeypatch):
    _fake_nvml(monkeypatch, [(1965, 0)])
    s = bench.ClockSampler(0)
    s.start()
    r = s.stop()
    assert r["samples"] >= 2 and r["sm_mhz"] == 1965.0 and r["reasons"] == []


def test_clock_sampler_flags_thermal_slowdown(monkeypatch):
    _fake_nvml(monkeypatch, [(1500, SW_POWER_CAP | SW_THERMAL)])
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.05)
    r = s.stop()
    assert r["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]


def test_clock_sampler_without_nvml(monkeypatch):
    _fake_nvml(monkeypatch, [(1965, 0)], fail=True)
    s = bench.ClockSampler(0)
    s.start()
    r = s.stop()
    assert r["reasons"] == ["NVML unavailable: RuntimeError"] and r["sm_mhz"] is None


def test_prompt_lengths_fixed_and_uniform():
    assert bench.prompt_lengths(4, 4096, "fixed") == [4096] * 4
    a = bench.prompt_lengths(256, 4096, "uniform", seed=0)
    assert len(a) == 256 and all(128 <= x <= 4096 for x in a)
    assert a == bench.prompt_lengths(256, 4096, "uniform", seed=0)  # seeded
    assert a != bench.prompt_lengths(256, 4096, "uniform", seed=1)  # per rank
    assert 1500 < sum(a) / len(a) < 2700  # mean of U[128, 4096] is 2112
    assert bench.prompt_lengths(3, 100, "uniform") == [100] * 3  # contexts below 128


def test_disagg_workload_names_the_baseline_config():
    w2 = bench.disagg_workload(1, 1, 64, 4096, "fixed")
    assert "1 attention + 1 FFN" in w2 and "batch 64" in w2 and w2.endswith("(BASELINE configs[1])")
    w8 = bench.disagg_workload(4, 4, 64, 4096, "uniform")
    assert "batch 256" in w8 and "uniform in [128, 4096]" in w8 and w8.endswith("(BASELINE configs[3])")
    assert "BASELINE" not in bench.disagg_workload(2, 2, 64, 4096, "fixed")  # no config has 2 + 2
