"""GPU parity of the reference-layout (drop-in) entry points through the C ABI.

Cases follow the reference's own CUDA tests (native/tests/progressive_gemv_test.cu):
golden prefixes 0..4 within 2e-4 + 2e-4*|e| (:243-262), one-hot inputs observe every
weight (:264-285), base-only / prefix-zero / bias-once contracts (:287-307), wide
reductions K = 257, 513, 4096 with 4x128 tiles (:430-450), raw FP16 scale bit patterns
0x0001 and 0x7BFF exactly (:452-495) and production-view validation (:497-632).
The exact-order decode and scalar-order linear must be bit-identical to the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import harpq_b200 as hqb  # noqa: E402
from conftest import SEEDED_NAMES, assert_close, device_stages, load_seeded, random_matrix  # noqa: E402
from oracle import oracle as orc  # noqa: E402


def _raw(m):
    codes, bits, f32 = device_stages(m)
    return hqb.RawMatrix(hqb.Geometry(*m.geometry), codes, bits, f32)


def test_golden_all_prefixes(native_golden, golden_matrix):
    rm = _raw(golden_matrix)
    bias = torch.from_numpy(native_golden["bias"]).cuda()
    for p in range(5):
        for b in range(2):
            x = torch.from_numpy(native_golden["inputs"][b]).cuda()
            y = rm.gemv(x, p, bias).cpu().numpy()
            assert_close(y, native_golden["prefix_outputs"][p][b], 2e-4, 2e-4, f"golden p{p} b{b}")


def test_golden_one_hot_observes_every_weight(native_golden, golden_matrix):
    rm = _raw(golden_matrix)
    cols = golden_matrix.cols
    for p in range(5):
        for c in range(cols):
            x = torch.zeros(cols, device="cuda")
            x[c] = 1.0
            y = rm.gemv(x, p).cpu().numpy()
            assert_close(y, native_golden["prefix_weights"][p][:, c], 2e-4, 2e-4, f"one-hot p{p} c{c}")


def test_base_only_prefix_zero_and_bias_once(native_golden, golden_matrix):
    base = orc.Matrix(golden_matrix.geometry, golden_matrix.codes[:1], golden_matrix.scales[:1])
    rm = _raw(base)
    x = torch.from_numpy(native_golden["inputs"][0]).cuda()
    bias = torch.from_numpy(native_golden["bias"]).cuda()
    assert_close(rm.gemv(x, 1, bias).cpu().numpy(), native_golden["prefix_outputs"][1][0], 2e-4, 2e-4, "base")
    assert torch.count_nonzero(rm.gemv(x, 0)).item() == 0
    assert torch.equal(rm.gemv(x, 0, bias), bias)


@pytest.mark.parametrize("cols", [257, 513, 4096])
def test_wide_reduction_strides(cols):
    rng = np.random.default_rng(cols)
    m = random_matrix(rng, 3, cols, tile=(4, 128), group=128)
    rm = _raw(m)
    x = ((np.arange(cols) % 29) - 14).astype(np.float32) / 32
    bias = np.array([0.125, -0.25, 0.375], np.float32)
    for p in range(5):
        y = rm.gemv(torch.from_numpy(x).cuda(), p, torch.from_numpy(bias).cuda()).cpu().numpy()
        assert_close(y, orc.linear_reference(m, x, p, bias)[0], 2e-4, 2e-4, f"K={cols} p{p}")


@pytest.mark.parametrize("geo", [((37, 70), (16, 32), 8), ((130, 259), (128, 128), 128), ((9, 33), (4, 8), 2),
                                 ((5, 7), (1, 1), 1)])
def test_generic_geometries(geo):
    shape, tile, group = geo
    rng = np.random.default_rng(sum(shape))
    m = random_matrix(rng, *shape, tile=tile, group=group)
    rm = _raw(m)
    x = rng.standard_normal(shape[1]).astype(np.float32)
    for p in range(5):
        y = rm.gemv(torch.from_numpy(x).cuda(), p).cpu().numpy()
        assert_close(y, orc.linear_reference(m, x, p)[0], 2e-4, 2e-4, f"{geo} p{p}")


def test_raw_fp16_scale_bit_patterns():
    g = hqb.Geometry(1, 1, 1, 1, 1, 1, 1)
    code = torch.tensor([1], dtype=torch.uint8, device="cuda")
    x = torch.tensor([1.0], device="cuda")
    for bits, want in ((0x0001, 2.0 ** -24), (0x7BFF, 65504.0)):
        s = torch.tensor([bits], dtype=torch.int32).to(torch.int16).cuda()
        y = hqb.RawMatrix(g, [code], [s]).gemv(x, 1)
        assert y.item() == want


def test_production_view_validation():
    g = hqb.geometry(5, 9, (4, 8), 4)
    codes = torch.zeros(32, dtype=torch.uint8, device="cuda")
    bits = torch.zeros(32, dtype=torch.int16, device="cuda")
    x = torch.zeros(9, device="cuda")
    y = torch.zeros(5, device="cuda")
    bias = torch.zeros(5, device="cuda")
    L = hqb.lib()
    st = (hqb.RawStage * 4)()
    st[0] = hqb.RawStage(codes.data_ptr(), 32, bits.data_ptr(), 32)

    def launch(prefix=1, xp=x, xc=9, bp=None, bc=0, yp=y, yc=5, stages=st, count=1, geo=g):
        import ctypes

        return L.hqb_raw_gemv(ctypes.byref(geo), stages, count, prefix, None if xp is None else xp.data_ptr(), xc,
                              None if bp is None else bp.data_ptr(), bc, None if yp is None else yp.data_ptr(), yc,
                              None)

    assert launch() == 0
    assert launch(bp=bias, bc=5, prefix=0) == 0
    torch.cuda.synchronize()
    assert launch(xp=None, yp=None) == 1
    assert launch(xc=8) == 1
    assert launch(yc=4) == 1
    assert launch(bp=bias, bc=0) == 1
    assert launch(bc=5) == 1
    assert launch(bp=bias, bc=4) == 1
    assert launch(prefix=2) == 1
    assert launch(count=0, prefix=0) == 1
    for field, value in (("packed_code_bytes", 31), ("scale_count", 31), ("packed_codes", None),
                         ("scale_fp16_bits", None)):
        bad = (hqb.RawStage * 4)()
        bad[0] = hqb.RawStage(codes.data_ptr(), 32, bits.data_ptr(), 32)
        setattr(bad[0], field, value)
        assert launch(stages=bad) == 1, field
    bad_geo = hqb.geometry(5, 9, (4, 8), 4)
    bad_geo.padded_columns = 15
    assert launch(geo=bad_geo) == 1


@pytest.mark.parametrize("name", SEEDED_NAMES)
def test_exact_order_decode_and_linear_are_bit_identical(name):
    m, _, z = load_seeded(name)
    rm = _raw(m)
    for p in range(5):
        assert rm.dequantize_prefix(p).cpu().numpy().tobytes() == orc.dequantize_prefix(m, p).tobytes()
        y = rm.linear_ordered(torch.from_numpy(z["x"]).cuda(), p, torch.from_numpy(z["bias"]).cuda())
        assert y.cpu().numpy().tobytes() == orc.linear_reference(m, z["x"], p, z["bias"]).tobytes()
    for s in range(4):
        assert rm.dequantize_stage(s).cpu().numpy().tobytes() == orc.dequantize_stage(m, s).tobytes()


def test_exact_order_golden(native_golden, golden_matrix):
    rm = _raw(golden_matrix)
    x = torch.from_numpy(native_golden["inputs"]).cuda()
    bias = torch.from_numpy(native_golden["bias"]).cuda()
    for p in range(5):
        assert rm.dequantize_prefix(p).cpu().numpy().tobytes() == native_golden["prefix_weights"][p].tobytes()
        y = rm.linear_ordered(x, p, bias).cpu().numpy()
        assert y.tobytes() == native_golden["prefix_outputs"][p].tobytes()


@pytest.mark.parametrize("name", SEEDED_NAMES)
def test_seeded_fixtures_raw_gemv(name):
    m, _, z = load_seeded(name)
    rm = _raw(m)
    for b in range(z["x"].shape[0]):
        for p in range(5):
            y = rm.gemv(torch.from_numpy(z["x"][b]).cuda(), p, torch.from_numpy(z["bias"]).cuda()).cpu().numpy()
            assert_close(y, orc.linear_reference(m, z["x"][b], p, z["bias"])[0], 2e-4, 2e-4, f"{name} b{b} p{p}")
