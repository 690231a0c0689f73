"""GPU: native C++ programs linked against libharpq_b200.so.

* harp-q_b200/lib/hqb_api_test — this repository's C++ API contract test.
* oracle/_ref/ref_*_test — the reference's own tests (native/tests/stage_codec_test.cpp,
  progressive_gemv_test.cu, cuda_oracle_test.cu) compiled unchanged against this
  repository's headers and library by oracle/build.py: the drop-in check of the
  native API.  They exist where the reference checkout was present at build time
  and travel with the working tree.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
REF_TESTS = ["ref_stage_codec_test", "ref_progressive_gemv_test", "ref_cuda_oracle_test"]


def _run(path: Path) -> subprocess.CompletedProcess:
    return subprocess.run([str(path)], capture_output=True, text=True, timeout=600)


def test_cpp_api_contract():
    exe = REPO / "harp-q_b200" / "lib" / "hqb_api_test"
    assert exe.exists(), "build() did not produce the C++ API test"
    r = _run(exe)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.parametrize("name", REF_TESTS)
def test_reference_suite_against_this_library(name):
    exe = REPO / "oracle" / "_ref" / name
    if not exe.exists():
        pytest.skip("reference test binaries were not built (no reference checkout at build time)")
    r = _run(exe)
    assert r.returncode == 0, r.stdout + r.stderr
