"""bench.py host logic without a GPU: the nvidia-smi clock sampler that runs
during the timed region (median SM clock, max clock, throttle reasons seen)."""
import os
import time

import bench

ROW = "0, {sm}, 1965, 700.5, 0x4, Not Active, Not Active, {thermal}, Active"


def _fake_smi(tmp_path, rows):
    fake = tmp_path / "nvidia-smi"
    lines = "".join(f"echo '{r}'; " for r in rows)
    fake.write_text(f"#!/bin/sh\nwhile true; do {lines}sleep 0.05; done\n")
    fake.chmod(0o755)
    return fake


def test_clock_sampler_reports_median_and_reasons(tmp_path, monkeypatch):
    _fake_smi(tmp_path, [ROW.format(sm=1965, thermal="Not Active"), ROW.format(sm=1800, thermal="Not Active")])
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.5)
    r = s.stop()
    assert r["samples"] >= 2
    assert r["sm_max_mhz"] == 1965.0
    assert 1800.0 <= r["sm_mhz"] <= 1965.0
    assert r["reasons"] == ["sw_power_cap"]  # power cap is kept and noted
    assert s.out is None and not s.path.exists()


def test_clock_sampler_flags_thermal_slowdown(tmp_path, monkeypatch):
    _fake_smi(tmp_path, [ROW.format(sm=1500, thermal="Active")])
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.3)
    r = s.stop()
    assert r["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]


def test_clock_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))  # an empty directory: no nvidia-smi
    s = bench.ClockSampler(0)
    s.start()
    r = s.stop()
    assert r["reasons"] == ["nvidia-smi unavailable"] and r["sm_mhz"] is None
    assert s.out is None and not s.path.exists()


def test_prompt_lengths_fixed_and_uniform():
    assert bench.prompt_lengths(4, 4096, "fixed") == [4096] * 4
    a = bench.prompt_lengths(256, 4096, "uniform", seed=0)
    assert len(a) == 256 and all(128 <= x <= 4096 for x in a)
    assert a == bench.prompt_lengths(256, 4096, "uniform", seed=0)  # seeded
    assert a != bench.prompt_lengths(256, 4096, "uniform", seed=1)  # per rank
    assert 1500 < sum(a) / len(a) < 2700  # mean of U[128, 4096] is 2112
    assert bench.prompt_lengths(3, 100, "uniform") == [100] * 3  # contexts below 128
