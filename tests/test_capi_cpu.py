"""CPU: the C-ABI library loads and exports every symbol include/harpq_b200.h declares;
host-only size queries and argument validation work without a GPU (no kernel runs)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "harpq_b200.h"
LIB = REPO / "harp-q_b200" / "lib" / "libharpq_b200.so"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"HQB_API\s+[\w\s\*]+?\b(hqb_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def hqb():
    if not LIB.exists():
        pytest.fail("libharpq_b200.so missing: run __graft_entry__.build()")
    import harpq_b200

    return harpq_b200


def test_every_declared_symbol_is_exported(hqb):
    names = declared_symbols()
    assert len(names) >= 19
    lib = ctypes.CDLL(str(LIB))
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(hqb.EXPORTS), "Python binding and header disagree"


def test_host_side_size_queries(hqb):
    L = hqb.lib()
    assert L.hqb_version() == 1
    g = hqb.geometry(11008, 4096)
    assert L.hqb_plane_bytes(ctypes.byref(g)) == 86 * 32 * 4352
    # 17*N*K/64 bytes per stage when N and K are tile multiples
    g = hqb.geometry(4096, 4096)
    assert L.hqb_plane_bytes(ctypes.byref(g)) == 17 * 4096 * 4096 // 64
    assert L.hqb_plane_bytes(ctypes.byref(hqb.geometry(100, 100, (4, 8), 4))) == 0
    bad = hqb.geometry(256, 256)
    bad.padded_rows = 300
    assert L.hqb_plane_bytes(ctypes.byref(bad)) == 0
    assert L.hqb_xfrag_bytes(4096, 1, hqb.F16) == 32 * 272
    assert L.hqb_xfrag_bytes(4096, 16, hqb.F32) == 32 * 16 * (512 + 8)
    assert L.hqb_xfrag_bytes(4096, 17, hqb.F16) == 0
    assert L.hqb_depth_plan_bytes(86) == 87 * 4


def test_validation_rejects_before_any_cuda_call(hqb):
    L = hqb.lib()
    # null matrix / bad batch / bad dtype are rejected with cudaErrorInvalidValue (1)
    assert L.hqb_gemv(None, 1, None, 1, 1, None, 0, None, 1, None, 0, None) == 1
    pm = hqb.PlaneMatrixC(100, 100, 1, 1, 1, 0, (ctypes.c_void_p * 4)())
    assert L.hqb_gemv_ex(ctypes.byref(pm), 1, None, None, 8, 1, 0, 0, None, 0, 16, 1, 256, 1 << 20, 0, None) == 1
    assert L.hqb_gemv_ex(ctypes.byref(pm), 2, None, None, 16, 1, 1, 0, None, 0, 16, 1, 256, 1 << 20, 0, None) == 1
    wrong_grid = hqb.PlaneMatrixC(300, 100, 1, 1, 1, 0, (ctypes.c_void_p * 4)())
    assert L.hqb_gemv_ex(ctypes.byref(wrong_grid), 1, None, None, 16, 1, 1, 0, None, 0, 16, 1, 256, 1 << 20, 0,
                         None) == 1
    st = hqb.RawStage(None, 0, None, 0)
    assert L.hqb_repack_stage(ctypes.byref(hqb.geometry(64, 64, (4, 8), 4)), ctypes.byref(st), 16, None, None) == 801
    assert L.hqb_repack_stage(ctypes.byref(hqb.geometry(128, 128)), ctypes.byref(st), 16, None, None) == 1
    # reference-layout view validation (progressive_gemv.cu:266-321)
    g = hqb.geometry(5, 9, (4, 8), 4)
    stages = (hqb.RawStage * 4)()
    assert L.hqb_raw_gemv(ctypes.byref(g), stages, 1, 2, 16, 9, None, 0, 32, 5, None) == 1  # prefix > count
    assert L.hqb_raw_gemv(ctypes.byref(g), stages, 1, 1, 16, 9, None, 0, 32, 5, None) == 1  # null stage storage
    assert L.hqb_raw_gemv(ctypes.byref(g), stages, 1, 0, 16, 8, None, 0, 32, 5, None) == 1  # short input
    assert L.hqb_raw_gemv(ctypes.byref(g), stages, 0, 0, 16, 9, None, 0, 32, 5, None) == 1  # no stages
    assert L.hqb_status_string(1).decode().startswith("invalid")
