"""ClockSampler (the clocks / throttle-reason record of every timed bench region),
parsed from a stand-in nvidia-smi that prints three samples: two under load with
the power cap active and one idle.  The median is taken over loaded samples only."""
import os
import stat
import time

from mtorus.utils.clocks import ClockSampler

_FAKE = """#!/bin/sh
echo "0, 1800, 1965, 950.5, 0x4, Not Active, Not Active, Not Active, Active"
echo "0, 1850, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active"
echo "0, 600, 1965, 100.0, 0x0, Not Active, Not Active, Not Active, Not Active"
exec sleep 30
"""


def test_sampler_parses_loaded_clocks_and_reasons(tmp_path, monkeypatch):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(_FAKE)
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    s = ClockSampler(gpu_index=0).start()
    time.sleep(0.5)
    r = s.stop()
    assert r["samples"] == 3
    assert r["sm_mhz"] == 1825.0 and r["sm_max_mhz"] == 1965.0 and r["power_w_max"] == 990.0
    assert r["reasons"] == ["sw_power_cap"]


def test_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    assert ClockSampler().start().stop()["reasons"] == ["nvidia-smi unavailable"]
