"""bench.py's clock sampler against a stand-in `nvidia-smi` on PATH (no GPU):
samples are collected even when the timed region is shorter than the tool's
start-up time, only samples from inside the region are kept, and throttle
reasons are reported by name."""

from __future__ import annotations

import stat
import sys
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _fake_smi(tmp_path: Path, reasons: str) -> None:
    script = tmp_path / "nvidia-smi"
    script.write_text(
        f"#!{sys.executable}\n"
        "import time\n"
        "time.sleep(0.15)  # start-up longer than the timed region\n"
        "while True:\n"
        f"    print('0, 1965, 1965, 500.0, 0x0, {reasons}', flush=True)\n"
        "    time.sleep(0.025)\n")
    script.chmod(script.stat().st_mode | stat.S_IXUSR)


@pytest.fixture
def bench_module(monkeypatch):
    monkeypatch.syspath_prepend(str(ROOT))
    import bench
    return bench


def test_short_region_gets_samples(tmp_path, monkeypatch, bench_module):
    _fake_smi(tmp_path, "Not Active, Not Active, Not Active, Not Active")
    monkeypatch.setenv("PATH", str(tmp_path))
    sampler = bench_module.ClockSampler(0)
    time.sleep(0.08)  # an 80 ms timed region
    info = sampler.stop()
    assert info["samples"] >= 1
    assert info["sm_mhz"] == 1965.0 and info["sm_max_mhz"] == 1965.0
    assert info["reasons"] == []


def test_throttle_reasons_are_reported(tmp_path, monkeypatch, bench_module):
    _fake_smi(tmp_path, "Not Active, Active, Not Active, Active")
    monkeypatch.setenv("PATH", str(tmp_path))
    sampler = bench_module.ClockSampler(0)
    time.sleep(0.05)
    info = sampler.stop()
    assert info["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]


def test_missing_tool_is_reported(tmp_path, monkeypatch, bench_module):
    monkeypatch.setenv("PATH", str(tmp_path))  # no nvidia-smi here
    info = bench_module.ClockSampler(0).stop()
    assert info["sm_mhz"] is None and info["reasons"] == ["nvidia-smi unavailable"]
