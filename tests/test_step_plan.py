"""Host-side check of the decode-step kernel's work partition (csrc/step_plan.h, shared
with the device code): builds tests/native/step_plan_check.cpp with the host compiler and
runs it. It checks that every (weight group, k block) cell of every projection is
multiplied by exactly one CTA, that ring slots are never overfilled, that pieces never
straddle a tile, that layer projections give a CTA at most two tiles (the TMEM budget)
and that every attention unit has exactly one owner."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_step_partition(tmp_path):
    exe = tmp_path / "step_plan_check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-o", str(exe), str(HERE / "native" / "step_plan_check.cpp")],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr
