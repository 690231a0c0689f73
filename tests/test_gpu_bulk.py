"""GPU parity of the bulk-copy GEMV (HQB_FLAG_BULK: plane chunks streamed into shared
memory by 1-D bulk copies, int8 activation limbs; batch <= 2, raw FP16/FP32 x).

Checked against the CPU oracle on the same seeded inputs: the scalar-order
ProgressiveLinearReference restatement within the reference's fused-GEMV tolerance
|a - e| <= 2e-4 + 2e-4*|e| (native/tests/progressive_gemv_test.cu:36-37) for plain x, the
FP64 materialize-then-matvec of the bit-exact decode for x with outlier channels (where the
oracle's own FP32 running sum drifts), and rel-L2 <= 2e-5 against FP64 always (the int8
form is exact up to the rounding of x to 30 bits of its tile's largest |x|).
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from conftest import assert_close, plane_matrix, random_matrix, rel_l2  # noqa: E402
from oracle import oracle as orc  # noqa: E402

FP16_RTOL = 2.0 ** -10


def _hqb():
    import harpq_b200 as hqb

    return hqb


def _fp64(m, x, prefix, bias=None, depth=None):
    w = orc.dequantize_prefix_np(m, prefix, depth=depth).astype(np.float64)
    y = np.asarray(x, np.float64).reshape(-1, m.cols) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    return y


def _case(rows, cols, batch, seed, outliers, stages=4):
    rng = np.random.default_rng(seed)
    m = random_matrix(rng, rows, cols, stages=stages)
    x = (rng.standard_normal((batch, cols)) * 2).astype(np.float16)
    if outliers:
        x[:, ::97] *= 20
    bias = rng.standard_normal(rows).astype(np.float32)
    return m, x, bias


@pytest.mark.parametrize("rows,cols", [(300, 520), (1000, 3000), (4096, 4096), (200, 11008), (65536, 256),
                                       (2048, 28672)])
@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("outliers", [False, True])
def test_bulk_kernel_against_oracle(rows, cols, batch, outliers):
    """Every prefix, FP32 and FP16 outputs, bias.  The shapes cover CTAs of a single chunk,
    chunks crossing tile rows, 86 and 224 tile columns (the latter with one activation
    preparation launch shared by all CTAs) and CTAs whose tiles wrap the two tile columns of
    65536x256 more than once."""
    hqb = _hqb()
    m, x, bias = _case(rows, cols, batch, rows + cols + batch, outliers)
    pm = plane_matrix(m)
    xt = torch.from_numpy(x).cuda()
    xf = x.astype(np.float32)
    bt = torch.from_numpy(bias).cuda()
    ws = pm.workspace(batch)
    fl = hqb.FLAG_BULK
    for p in (1, 2, 3, 4):
        assert pm.gemv_kernel(batch, hqb.F16, p, flags=fl) == "gemv_bulk_kernel"
        y = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float32, workspace=ws, flags=fl).cpu().numpy()
        e64 = _fp64(m, xf, p, bias)
        # the scalar-order oracle's own FP32 running sum drifts past the contract with outlier
        # channels or beyond ~11k columns: FP64 there
        want = e64 if outliers or cols > 11008 else orc.linear_reference(m, xf, p, bias)
        assert_close(y, want, 2e-4, 2e-4, f"{rows}x{cols} b{batch} p{p}")
        assert rel_l2(y, e64) <= 2e-5, f"{rows}x{cols} b{batch} p{p} rel-L2 {rel_l2(y, e64):.2e}"
        y16 = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float16, workspace=ws, flags=fl).float().cpu().numpy()
        assert_close(y16, e64, 2e-4, FP16_RTOL, f"{rows}x{cols} b{batch} p{p} f16")
    assert ws.error_flags() == 0


@pytest.mark.parametrize("batch", [1, 2])
def test_bulk_kernel_fp32_activations(batch):
    """FP32 x (limbs built from FP32 values) spanning 1e-6..1e6 inside every tile, checked
    element by element: each x keeps at least 24 bits relative to its tile's largest |x|,
    so the error of an output is bounded by sum_c |w_c| * 2^-23 * max|x| of c's tile."""
    hqb = _hqb()
    rng = np.random.default_rng(17 + batch)
    m = random_matrix(rng, 640, 1000)
    pm = plane_matrix(m)
    mag = 10.0 ** rng.uniform(-6, 6, size=(batch, m.cols))
    x = (np.sign(rng.standard_normal((batch, m.cols))) * mag).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    for p in (1, 4):
        y = pm.gemv(xt, prefix=p, y_dtype=torch.float32, flags=hqb.FLAG_BULK).cpu().numpy()
        w = orc.dequantize_prefix_np(m, p).astype(np.float64)
        e64 = x.astype(np.float64) @ w.T
        tile_max = np.abs(x).reshape(batch, -1)
        pad = (-m.cols) % 128
        tm = np.pad(tile_max, ((0, 0), (0, pad))).reshape(batch, -1, 128).max(-1)
        per_col = np.repeat(tm, 128, axis=1)[:, :m.cols]
        bound = (np.abs(w)[None, :, :] * per_col[:, None, :]).sum(-1) * 2.0 ** -23 + 1e-30
        err = np.abs(y - e64)
        assert np.all(err <= 4 * bound), f"p{p}: worst ratio {(err / bound).max():.2f}"
        assert rel_l2(y, e64) <= 1e-5


@pytest.mark.parametrize("batch", [1, 2])
def test_bulk_kernel_nonfinite_and_huge_activations(batch):
    """A NaN activation makes every output of its batch row NaN (as the reference's FP32
    sum does); an Inf activation too (the reference gives +-Inf or NaN row by row; this
    kernel gives NaN); finite activations up to 1e35 (beyond 2^100, the wide-tile factor)
    give the FP64 result within the FP32 contract."""
    hqb = _hqb()
    rng = np.random.default_rng(5 + batch)
    m = random_matrix(rng, 512, 768)
    pm = plane_matrix(m)
    w = orc.dequantize_prefix_np(m, 3).astype(np.float64)
    # huge finite values in one tile of row 0
    x = (rng.standard_normal((batch, m.cols))).astype(np.float32)
    x[0, 130:140] = 1e35
    x[0, 200] = -3e34
    y = pm.gemv(torch.from_numpy(x).cuda(), prefix=3, y_dtype=torch.float32, flags=hqb.FLAG_BULK).cpu().numpy()
    e64 = x.astype(np.float64) @ w.T
    assert np.all(np.isfinite(y))
    # row 0: each x keeps 24 bits of its tile's largest |x| (1e35 in the huge tile)
    bound = np.abs(w) @ np.full(m.cols, 1e35) * 2.0 ** -22
    assert np.all(np.abs(y[0] - e64[0]) <= bound), "huge x"
    assert rel_l2(y[0], e64[0]) <= 1e-5
    if batch == 2:
        assert_close(y[1], e64[1], 2e-4, 2e-4, "ordinary row next to the huge one")
    for bad in (np.nan, np.inf):
        xb = x.copy()
        xb[0, 130:140] = 1.0
        xb[0, 200] = 1.0
        xb[0, 333] = bad
        y = pm.gemv(torch.from_numpy(xb).cuda(), prefix=3, y_dtype=torch.float32, flags=hqb.FLAG_BULK).cpu().numpy()
        assert np.all(np.isnan(y[0])), f"{bad}: batch row 0 must be NaN"
        if batch == 2:
            e1 = xb[1].astype(np.float64) @ w.T
            assert np.all(np.isfinite(y[1]))
            assert rel_l2(y[1], e1) <= 2e-5


@pytest.mark.parametrize("rows,cols", [(300, 520), (11008, 4096), (200, 11008)])
@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("x_dtype", ["f16", "f32"])
def test_bulk_kernel_depth_map(rows, cols, batch, x_dtype):
    """A per-tile depth map on the bulk kernel: the scalar-order oracle (linear_mixed) for
    FP16-exact x, FP64 within 2e-5 rel-L2, repeatable bytes.  11008x4096 with the map of
    seed 7 is the mixed-depth configuration."""
    hqb = _hqb()
    m, x, bias = _case(rows, cols, batch, rows + 5 * cols + batch, False)
    pm = plane_matrix(m)
    gr, gc = m.grid
    depth = np.random.default_rng(7).integers(1, 5, size=(gr, gc)).astype(np.uint8)
    plan = hqb.DepthPlan(torch.from_numpy(depth).cuda(), pm.stage_count)
    xf = x.astype(np.float32)
    xt = torch.from_numpy(x).cuda() if x_dtype == "f16" else torch.from_numpy(xf).cuda()
    bt = torch.from_numpy(bias).cuda()
    ws = pm.workspace(batch, hqb.F32)
    fl = hqb.FLAG_BULK
    assert pm.gemv_kernel(batch, hqb.F16 if x_dtype == "f16" else hqb.F32, 0, mixed=True, flags=fl) == \
        "gemv_bulk_kernel"
    y = pm.gemv(xt, depth=plan, bias=bt, y_dtype=torch.float32, workspace=ws, flags=fl)
    y2 = pm.gemv(xt, depth=plan, bias=bt, y_dtype=torch.float32, workspace=ws, flags=fl)
    assert torch.equal(y, y2)
    y = y.cpu().numpy()
    e64 = _fp64(m, xf, 4, bias, depth=depth)
    assert_close(y, orc.linear_mixed(m, xf, depth, bias), 2e-4, 2e-4, f"{rows}x{cols} b{batch}")
    assert rel_l2(y, e64) <= 2e-5
    assert ws.error_flags() == 0


def test_bulk_matches_register_ring_kernel_and_pdl():
    """Same limb slots and the same partition arithmetic as the register-ring stream-K
    kernel: equal within the FP32 contract (the stream-K grid and summation order may
    differ); programmatic-dependent launches give the same bytes as plain launches."""
    hqb = _hqb()
    rng = np.random.default_rng(99)
    m = random_matrix(rng, 3000, 2000)
    pm = plane_matrix(m)
    x = torch.from_numpy((rng.standard_normal((2, m.cols)) * 3).astype(np.float16)).cuda()
    ws = pm.workspace(2)
    for p in (1, 2, 3, 4):
        a = pm.gemv(x, prefix=p, y_dtype=torch.float32, workspace=ws, flags=hqb.FLAG_BULK)
        b = pm.gemv(x, prefix=p, y_dtype=torch.float32, workspace=ws, flags=hqb.FLAG_BULK | hqb.FLAG_PDL)
        c = pm.gemv(x, prefix=p, y_dtype=torch.float32, workspace=ws, flags=hqb.FLAG_STREAMK)
        torch.cuda.synchronize()
        assert torch.equal(a, b), p
        assert_close(a.cpu().numpy(), c.cpu().numpy(), 2e-4, 2e-4, f"bulk vs stream-K p{p}")
    assert ws.error_flags() == 0
