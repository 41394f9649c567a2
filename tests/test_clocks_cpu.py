"""Clock sampler on CPU: a stand-in ``nvidia-smi`` on PATH writes the CSV rows."""

from __future__ import annotations

import os
import stat
import time

from conftest import mod

FAKE = """#!/bin/sh
echo "0, 1965, 1965, 650.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active"
echo "0, 1800, 1965, 990.4, 0x0000000000000004, Not Active, Not Active, Not Active, Active"
echo "0, 1900, 1965, 980.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active"
exec sleep 10
"""


def test_sampler_summarizes_clocks_and_reasons(tmp_path, monkeypatch):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE)
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ.get('PATH', '')}")
    clocks = mod("utils.clocks")
    with clocks.ClockSampler(0, period_ms=50) as s:
        time.sleep(0.5)
    out = s.summary()
    assert out["samples"] == 3
    assert out["sm_mhz"] == 1900.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]
    assert out["power_w_max"] == 990.4


def test_sampler_without_nvidia_smi_reports_unsampled(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    clocks = mod("utils.clocks")
    with clocks.ClockSampler(0) as s:
        pass
    assert s.summary()["reasons"] == ["unsampled"]
