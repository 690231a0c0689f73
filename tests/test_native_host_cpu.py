"""CPU: the reference's host functions through this library without a GPU.

DequantizeStage, DequantizePrefix and ProgressiveLinearReference are host functions in
the reference (native/src/stage_codec.cpp:225-339) and its CPU CI runs their tests
(native/tests/stage_codec_test.cpp).  This library runs them on the device when one is
usable and as host loops of the same FP32 operations otherwise.  Here the reference's own
stage-codec test program, compiled unchanged against this library by oracle/build.py,
runs with every device hidden, so the host forms are what it checks.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def test_reference_stage_codec_suite_without_a_device():
    exe = REPO / "oracle" / "_ref" / "ref_stage_codec_test"
    if not exe.exists():
        pytest.skip("reference test binaries were not built (no reference checkout at build time)")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
