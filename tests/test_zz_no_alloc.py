"""hqb_gemv_noalloc: the GEMV with the library's fixed per-device scratch.

Collected last (file name) so that it also runs after every other GPU test in the same
process.  Each case calls the entry point twice in a row through the C ABI and checks
both results against hqb_gemv with a caller-owned workspace, on the same inputs:
FP32 outputs within 2e-4 + 2e-4*|e|, FP16 outputs within 2e-4 + 2^-10*|e|.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from conftest import SEEDED_NAMES, assert_close, load_seeded, plane_matrix, random_matrix  # noqa: E402

FP16_RTOL = 2.0 ** -10


def _lib():
    import harpq_b200 as hqb

    return hqb, hqb.lib()


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _both(pm, x, prefix, bias, y_dtype):
    """(hqb_gemv with a workspace, first noalloc call, second noalloc call)."""
    hqb, L = _lib()
    xd = hqb.F32 if x.dtype == torch.float32 else hqb.F16
    yd = hqb.F32 if y_dtype == torch.float32 else hqb.F16
    bd = hqb.F32 if bias is None or bias.dtype == torch.float32 else hqb.F16
    batch = x.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    ws = pm.workspace(batch, xd)
    m = pm.c_struct()
    outs = []
    y = torch.full((batch, pm.rows), float("nan"), dtype=y_dtype, device="cuda")
    st = L.hqb_gemv(ctypes.byref(m), prefix, _ptr(x), xd, batch, _ptr(bias), bd, _ptr(y), yd, ws.ptr(), ws.nbytes,
                    stream)
    assert st == 0, st
    outs.append(y)
    for _ in range(2):
        y = torch.full((batch, pm.rows), float("nan"), dtype=y_dtype, device="cuda")
        st = L.hqb_gemv_noalloc(ctypes.byref(m), prefix, _ptr(x), xd, batch, _ptr(bias), bd, _ptr(y), yd, stream)
        assert st == 0, (st, L.hqb_status_string(st))
        outs.append(y)
    torch.cuda.synchronize()
    return [o.float().cpu().numpy() for o in outs]


def _check(ref, got, y_dtype, what):
    rtol = 2e-4 if y_dtype == torch.float32 else FP16_RTOL
    assert_close(got, ref, 2e-4, rtol, what)


@pytest.mark.gpu
@pytest.mark.parametrize("name", SEEDED_NAMES)
@pytest.mark.parametrize("y_dtype", [torch.float32, torch.float16])
def test_noalloc_matches_gemv_seeded(name, y_dtype):
    m, _, z = load_seeded(name)
    pm = plane_matrix(m)
    x = torch.from_numpy(z["x"]).cuda().half()
    bias = torch.from_numpy(z["bias"]).cuda()
    for p in (1, 2, 3, 4):
        ref, a, b = _both(pm, x, p, bias, y_dtype)
        _check(ref, a, y_dtype, f"{name} p{p} first call")
        _check(ref, b, y_dtype, f"{name} p{p} second call")


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 4])
@pytest.mark.parametrize("x_dtype", [torch.float16, torch.float32])
def test_noalloc_matches_gemv_layer(batch, x_dtype):
    rng = np.random.default_rng(7 + batch)
    m = random_matrix(rng, 1000, 4100)
    pm = plane_matrix(m)
    x = torch.from_numpy(rng.standard_normal((batch, m.cols)).astype(np.float32)).cuda().to(x_dtype)
    for p in (1, 3):
        ref, a, b = _both(pm, x, p, None, torch.float32)
        _check(ref, a, torch.float32, f"batch {batch} p{p} first call")
        _check(ref, b, torch.float32, f"batch {batch} p{p} second call")


@pytest.mark.gpu
def test_noalloc_rejects_work_beyond_the_scratch():
    hqb, L = _lib()
    rng = np.random.default_rng(11)
    m = random_matrix(rng, 256, 512)
    pm = plane_matrix(m)
    batch = 16
    need = L.hqb_workspace_bytes(ctypes.byref(pm.c_struct()), batch, hqb.F32, torch.cuda.current_device())
    assert need > hqb.NOALLOC_SCRATCH_BYTES
    x = torch.ones(batch, m.cols, device="cuda")
    y = torch.full((batch, m.rows), 7.0, device="cuda")
    st = L.hqb_gemv_noalloc(ctypes.byref(pm.c_struct()), 2, _ptr(x), hqb.F32, batch, None, hqb.F32, _ptr(y), hqb.F32,
                            torch.cuda.current_stream().cuda_stream)
    assert st == hqb.ERR_SCRATCH_LIMIT
    assert b"HQB_NOALLOC_SCRATCH_BYTES" in L.hqb_status_string(st)
    torch.cuda.synchronize()
    assert bool((y == 7.0).all()), "a rejected call wrote its output"


@pytest.mark.gpu
def test_noalloc_invalid_arguments():
    hqb, L = _lib()
    rng = np.random.default_rng(12)
    pm = plane_matrix(random_matrix(rng, 128, 128, stages=2))
    x = torch.ones(1, 128, device="cuda", dtype=torch.float16)
    y = torch.empty(1, 128, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    m = pm.c_struct()
    assert L.hqb_gemv_noalloc(None, 1, _ptr(x), hqb.F16, 1, None, hqb.F32, _ptr(y), hqb.F32, s) == 1
    assert L.hqb_gemv_noalloc(ctypes.byref(m), 3, _ptr(x), hqb.F16, 1, None, hqb.F32, _ptr(y), hqb.F32, s) == 1
    assert L.hqb_gemv_noalloc(ctypes.byref(m), 1, _ptr(x), hqb.F16, 0, None, hqb.F32, _ptr(y), hqb.F32, s) == 1
    assert L.hqb_gemv_noalloc(ctypes.byref(m), 1, _ptr(x), 7, 1, None, hqb.F32, _ptr(y), hqb.F32, s) == 1


@pytest.mark.gpu
def test_noalloc_error_word_read_clear_and_reset():
    """The scratch's error word through the C ABI: a set bit is read back by
    hqb_gemv_noalloc_flags (and cleared on request); hqb_gemv_noalloc_reset returns the whole
    array to its first-call state, after which the GEMV matches hqb_gemv again."""
    hqb, L = _lib()
    rng = np.random.default_rng(404)
    m = random_matrix(rng, 700, 900)
    pm = plane_matrix(m)
    x = torch.from_numpy(rng.standard_normal((1, m.cols)).astype(np.float16)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    ref, a, b = _both(pm, x, 3, None, torch.float32)
    flags = ctypes.c_int(-1)
    assert L.hqb_gemv_noalloc_flags(ctypes.byref(flags), 0, stream) == 0
    assert flags.value == 0
    # set the error word as a kernel would after a bounded wait ran out
    addr = ctypes.c_void_p()
    assert L.hqb_gemv_noalloc_scratch(ctypes.byref(addr)) == 0
    word = torch.as_tensor(hqb._DeviceView(addr.value, (1,), "<i4"), device="cuda")
    word.fill_(hqb.DEVERR_TIMEOUT)
    torch.cuda.synchronize()
    assert L.hqb_gemv_noalloc_flags(ctypes.byref(flags), 0, stream) == 0
    assert flags.value == hqb.DEVERR_TIMEOUT
    assert L.hqb_gemv_noalloc_flags(ctypes.byref(flags), 1, stream) == 0  # read and clear
    assert flags.value == hqb.DEVERR_TIMEOUT
    assert L.hqb_gemv_noalloc_flags(ctypes.byref(flags), 0, stream) == 0
    assert flags.value == 0
    # a damaged scratch (non-zero split-row words) is repaired by the reset
    word.fill_(hqb.DEVERR_TIMEOUT)
    assert L.hqb_gemv_noalloc_reset(stream) == 0
    assert L.hqb_gemv_noalloc_flags(ctypes.byref(flags), 0, stream) == 0
    assert flags.value == 0
    ref2, a2, b2 = _both(pm, x, 3, None, torch.float32)
    for got in (a, b, a2, b2):
        _check(ref, got, torch.float32, "noalloc after reset")
