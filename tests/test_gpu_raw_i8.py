"""GPU parity of raw_i8_kernel, the int8-limb kernel behind hqb_raw_gemv /
LaunchProgressiveGemv for 128x128 tiles with group 128 (reference
native/src/progressive_gemv.cu:420-439 is the entry it serves).

It reads the reference's row-major codes and FP16 scales in place.  The bar is the
reference's own fused-GEMV tolerance, 2e-4 + 2e-4*|expected| against the scalar-order
ProgressiveLinearReference restatement (native/tests/progressive_gemv_test.cu:36-37,
207-226), at sizes the oracle finishes quickly; at full layer sizes an FP64 product
of the exact decoded weights, by relative L2 and elementwise error bounds.  Also: the
kernel choice (HQB_RAW_REQUIRE_FAST / HQB_RAW_GENERIC), bit-identical repeats, ragged
shapes, unsupported geometries and misaligned code arrays falling back, and FP32
activations far outside the usual range.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import harpq_b200 as hqb  # noqa: E402
from conftest import assert_close, device_stages, random_matrix, rel_l2  # noqa: E402
from oracle import oracle as orc  # noqa: E402

TOL = 2e-4  # reference progressive_gemv_test.cu:36-37


def _raw(m):
    codes, bits, f32 = device_stages(m)
    return hqb.RawMatrix(hqb.Geometry(*m.geometry), codes, bits, f32)


def _tile_max(x):
    """Each column's 128-column tile maximum |x|: every activation keeps 24 bits or more
    of it in the int8 limbs, so |error| <= sum |w| * tile max * 2^-22 bounds a row."""
    xa = np.abs(np.asarray(x, np.float64))
    pad = -len(xa) % 128
    t = np.pad(xa, (0, pad)).reshape(-1, 128).max(axis=1)
    return np.repeat(t, 128)[: len(xa)]


def _fp64(m, x, prefix, bias=None):
    w = orc.dequantize_prefix_np(m, prefix).astype(np.float64)
    y = w @ np.asarray(x, np.float64)
    return y if bias is None else y + np.asarray(bias, np.float64)


@pytest.mark.parametrize("rows,cols", [(128, 128), (300, 520), (1000, 1100), (129, 4096), (2048, 1027)])
def test_fast_kernel_against_scalar_oracle(rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    m = random_matrix(rng, rows, cols)
    rm = _raw(m)
    x = rng.standard_normal(cols).astype(np.float32)
    bias = rng.standard_normal(rows).astype(np.float32)
    xt, bt = torch.from_numpy(x).cuda(), torch.from_numpy(bias).cuda()
    for p in range(1, 5):
        for b in (None, bt):
            y = rm.gemv(xt, p, b, flags=hqb.RAW_REQUIRE_FAST).cpu().numpy()
            e = orc.linear_reference(m, x, p, None if b is None else bias)[0]
            assert_close(y, e, TOL, TOL, f"{rows}x{cols} p{p} bias={b is not None}")
            g = rm.gemv(xt, p, b, flags=hqb.RAW_GENERIC).cpu().numpy()
            assert_close(y, g, TOL, TOL, f"fast vs generic {rows}x{cols} p{p}")


def test_fast_kernel_is_default_and_bit_repeatable():
    rng = np.random.default_rng(11)
    m = random_matrix(rng, 700, 900)
    rm = _raw(m)
    xt = torch.from_numpy(rng.standard_normal(900).astype(np.float32)).cuda()
    first = rm.gemv(xt, 3)
    assert torch.equal(first, rm.gemv(xt, 3, flags=hqb.RAW_REQUIRE_FAST))
    for _ in range(3):
        assert torch.equal(first, rm.gemv(xt, 3))


@pytest.mark.parametrize("rows,cols,prefix", [(4096, 4096, 2), (11008, 4096, 3), (4096, 11008, 4), (2048, 28672, 1)])
def test_fast_kernel_full_layer_sizes(rows, cols, prefix):
    rng = np.random.default_rng(rows + cols + prefix)
    m = random_matrix(rng, rows, cols, stages=prefix)
    rm = _raw(m)
    x = rng.standard_normal(cols).astype(np.float32)
    y = rm.gemv(torch.from_numpy(x).cuda(), prefix, flags=hqb.RAW_REQUIRE_FAST).cpu().numpy()
    e = _fp64(m, x, prefix)
    assert rel_l2(y, e) <= 5e-6
    w_abs = np.abs(orc.dequantize_prefix_np(m, prefix).astype(np.float64))
    assert np.all(np.abs(y - e) <= w_abs @ _tile_max(x) * 2.0 ** -22)


def test_unsupported_geometry_and_misaligned_codes_fall_back():
    rng = np.random.default_rng(5)
    # 64-wide tiles: not the fast kernel's geometry
    m = random_matrix(rng, 200, 300, tile=(64, 64), group=64)
    rm = _raw(m)
    x = rng.standard_normal(300).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    with pytest.raises(hqb.HQBError) as ei:
        rm.gemv(xt, 2, flags=hqb.RAW_REQUIRE_FAST)
    assert ei.value.status == hqb.HQB_ERR_UNSUPPORTED
    assert_close(rm.gemv(xt, 2).cpu().numpy(), orc.linear_reference(m, x, 2)[0], TOL, TOL, "64x64 default")
    # 128x128 geometry with a code array that starts 4 bytes past an 8-byte boundary
    m = random_matrix(rng, 256, 384)
    codes, bits, f32 = device_stages(m)
    shifted = []
    for c in codes:
        buf = torch.zeros(c.numel() + 4, dtype=torch.uint8, device="cuda")
        buf[4:] = c
        shifted.append(buf[4:])
    assert shifted[0].data_ptr() % 8 == 4
    rm = hqb.RawMatrix(hqb.Geometry(*m.geometry), shifted, bits, f32)
    x = rng.standard_normal(384).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    with pytest.raises(hqb.HQBError) as ei:
        rm.gemv(xt, 2, flags=hqb.RAW_REQUIRE_FAST)
    assert ei.value.status == hqb.HQB_ERR_UNSUPPORTED
    assert_close(rm.gemv(xt, 2).cpu().numpy(), orc.linear_reference(m, x, 2)[0], TOL, TOL, "misaligned default")
    with pytest.raises(hqb.HQBError):
        rm.gemv(xt, 2, flags=hqb.RAW_GENERIC | hqb.RAW_REQUIRE_FAST)


def test_prefix_zero_is_bias_or_zero():
    rng = np.random.default_rng(9)
    m = random_matrix(rng, 256, 256)
    rm = _raw(m)
    xt = torch.from_numpy(rng.standard_normal(256).astype(np.float32)).cuda()
    bt = torch.from_numpy(rng.standard_normal(256).astype(np.float32)).cuda()
    assert torch.equal(rm.gemv(xt, 0, bt), bt)
    assert torch.count_nonzero(rm.gemv(xt, 0)).item() == 0


def test_fp32_activations_wide_range_and_non_finite():
    rng = np.random.default_rng(21)
    rows, cols = 640, 1300
    m = random_matrix(rng, rows, cols)
    rm = _raw(m)
    w = orc.dequantize_prefix_np(m, 4).astype(np.float64)
    # magnitudes spanning 1e-30 .. 1e35 (a tile above 2^100 takes the wide-factor epilogue)
    x = (rng.standard_normal(cols) * 10.0 ** rng.uniform(-30, 6, cols)).astype(np.float32)
    x[700] = 1e35
    y = rm.gemv(torch.from_numpy(x).cuda(), 4, flags=hqb.RAW_REQUIRE_FAST).cpu().numpy().astype(np.float64)
    e = w @ x.astype(np.float64)
    assert np.all(np.isfinite(y))
    assert np.all(np.abs(y - e) <= np.abs(w) @ _tile_max(x) * 2.0 ** -22)
    # a NaN or Inf activation makes every output non-finite, as the reference's FMAs do
    for bad in (np.nan, np.inf):
        xb = x.copy()
        xb[3] = bad
        yb = rm.gemv(torch.from_numpy(xb).cuda(), 4, flags=hqb.RAW_REQUIRE_FAST).cpu().numpy()
        assert not np.any(np.isfinite(yb))
