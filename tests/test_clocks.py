"""The clock sampler against a fake nvidia-smi (no GPU): samples stamped
inside the timed region are kept, and a region shorter than the polling
interval still reports one sample."""
from __future__ import annotations

import os
import stat
import time

from gpu_mesh_b200.clocks import ClockSampler

FAKE = """#!/bin/sh
sleep 0.3
i=0
while [ $i -lt 400 ]; do
  echo "0, 1965, 1965, 700.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active"
  sleep 0.05
  i=$((i+1))
done
"""


def fake_smi(tmp_path, monkeypatch):
    path = tmp_path / "nvidia-smi"
    path.write_text(FAKE)
    path.chmod(path.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")


def test_samples_inside_the_region(tmp_path, monkeypatch):
    fake_smi(tmp_path, monkeypatch)
    with ClockSampler(0) as c:
        time.sleep(0.5)
    s = c.summary()
    assert s["samples"] >= 4
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]


def test_short_region_still_has_a_sample(tmp_path, monkeypatch):
    fake_smi(tmp_path, monkeypatch)
    with ClockSampler(0) as c:
        pass
    assert c.summary()["samples"] >= 1


def test_missing_nvidia_smi_reports_no_samples(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    with ClockSampler(0) as c:
        pass
    assert c.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
