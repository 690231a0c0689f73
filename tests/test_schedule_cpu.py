"""CPU: the work partition shared by host and device code (hqb_schedule.h), compiled
with the host compiler and checked exhaustively on random shapes and weights."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def test_partition_ranges_and_owner(tmp_path):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no host C++ compiler")
    exe = tmp_path / "partition_test"
    subprocess.run([cxx, "-std=c++17", "-O2", "-I", str(REPO / "harp-q_b200" / "csrc"),
                    str(REPO / "tests" / "native" / "partition_test.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "partition ok" in out.stdout
