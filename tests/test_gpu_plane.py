"""GPU parity of the plane-layout path (repack, bit-exact decode, tensor-core GEMV).

Every case is checked against the CPU oracle on the same seeded inputs:
* decode: bit-identical to the oracle's DequantizePrefix restatement;
* GEMV, FP32 outputs: |a - e| <= 2e-4 + 2e-4*|e| against the oracle's scalar-order
  ProgressiveLinearReference (the reference's fused-GEMV contract,
  native/tests/progressive_gemv_test.cu:36-37, docs/DECISIONS.md D-019), and
  rel-L2 <= 1e-3 against an FP64 materialize-then-matvec of the exact decoded weights;
* GEMV, FP16 outputs: |a - e| <= 2e-4 + 2^-10*|e| against that FP64 result (one FP16
  rounding of the output on top of the FP32 contract), rel-L2 <= 1e-3.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from conftest import (SEEDED_NAMES, assert_close, load_seeded, plane_matrix, random_matrix,  # noqa: E402
                      rel_l2)
from oracle import oracle as orc  # noqa: E402

FP16_RTOL = 2.0 ** -10


def _fp64_reference(m, x, prefix, bias=None, depth=None):
    w = orc.dequantize_prefix_np(m, prefix, depth=depth).astype(np.float64)
    y = np.asarray(x, np.float64).reshape(-1, m.cols) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    return y


@pytest.mark.parametrize("name", SEEDED_NAMES)
def test_plane_decode_bit_exact(name):
    m, _, _ = load_seeded(name)
    pm = plane_matrix(m)
    for p in range(5):
        got = pm.decode(p).cpu().numpy()
        assert got.tobytes() == orc.dequantize_prefix(m, p).tobytes(), f"prefix {p}"
    assert int(pm.repack_flags.item()) == 0


@pytest.mark.parametrize("name", SEEDED_NAMES)
@pytest.mark.parametrize("y_dtype", ["f32", "f16"])
def test_gemv_seeded_against_oracle(name, y_dtype):
    m, _, z = load_seeded(name)
    pm = plane_matrix(m)
    x = z["x"]  # FP16-exact activations, [batch, cols]
    bias = z["bias"]
    xt = torch.from_numpy(x).cuda().half()
    bt = torch.from_numpy(bias).cuda()
    ydt = torch.float32 if y_dtype == "f32" else torch.float16
    for p in range(5):
        y = pm.gemv(xt, prefix=p, bias=bt, y_dtype=ydt).float().cpu().numpy()
        e64 = _fp64_reference(m, x, p, bias)
        if y_dtype == "f32":
            scalar = orc.linear_reference(m, x, p, bias)
            assert_close(y, scalar, 2e-4, 2e-4, f"{name} p{p} vs scalar oracle")
        else:
            assert_close(y, e64, 2e-4, FP16_RTOL, f"{name} p{p} f16")
        assert rel_l2(y, e64) <= 1e-3


@pytest.mark.parametrize("batch", [1, 2, 5, 8, 9, 16])
@pytest.mark.parametrize("x_dtype", ["f16", "f32"])
def test_gemv_batches_and_dtypes(batch, x_dtype):
    rng = np.random.default_rng(100 + batch)
    m = random_matrix(rng, 300, 520)
    pm = plane_matrix(m)
    x = rng.standard_normal((batch, m.cols)).astype(np.float32) * 3
    if x_dtype == "f16":
        x = x.astype(np.float16).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    xt = xt.half() if x_dtype == "f16" else xt
    bias = rng.standard_normal(m.rows).astype(np.float32)
    bt = torch.from_numpy(bias).cuda().half()
    for p in (1, 2, 3, 4):
        y = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float32).cpu().numpy()
        e64 = _fp64_reference(m, x, p, bias.astype(np.float16).astype(np.float32))
        assert_close(y, e64, 2e-4, 2e-4, f"b{batch} {x_dtype} p{p}")
        assert rel_l2(y, e64) <= 1e-3


def test_fp32_activations_wide_dynamic_range():
    """FP32 x spanning 1e-6..1e6 in every tile (int8 limbs at batch 2: each x keeps at least
    24 bits relative to its tile's largest |x|)."""
    rng = np.random.default_rng(7)
    m = random_matrix(rng, 256, 384)
    mag = 10.0 ** rng.uniform(-6, 6, size=(2, m.cols))
    x = (np.sign(rng.standard_normal((2, m.cols))) * mag).astype(np.float32)
    # rows whose codes are zero at the tile's largest columns depend on the small activations
    for r in range(0, m.rows, 7):
        for s in range(4):
            c0 = int(np.argmax(np.abs(x[0, :128])))
            byte, sh = divmod(r * m.geometry[3] + c0, 4)
            m.codes[s][byte] &= np.uint8(~(3 << (2 * sh)) & 0xFF)
    pm = plane_matrix(m)
    y = pm.gemv(torch.from_numpy(x).cuda(), prefix=4, y_dtype=torch.float32).cpu().numpy()
    e64 = _fp64_reference(m, x, 4)
    assert rel_l2(y, e64) <= 1e-5
    # element by element: every x keeps >= 24 bits of its 128-column tile's largest |x|
    # (2^-24 of it), and the FP32 sums of 3 tiles x 4 stages add at most 12 roundings of
    # 2^-24 of the same magnitude: sum_c |w_rc| * tile max * 2^-20 bounds a row
    w = np.abs(orc.dequantize_prefix_np(m, 4).astype(np.float64))
    xa = np.abs(x.astype(np.float64))
    tmax = np.repeat(np.pad(xa, ((0, 0), (0, -m.cols % 128))).reshape(2, -1, 128).max(axis=2), 128, axis=1)[:, :m.cols]
    bound = tmax @ w.T * 2.0 ** -20
    assert np.all(np.abs(y - e64) <= bound)


def test_prefix_zero_writes_bias_or_zeros():
    rng = np.random.default_rng(1)
    m = random_matrix(rng, 200, 130)
    pm = plane_matrix(m)
    x = torch.randn(3, m.cols, device="cuda").half()
    y = pm.gemv(x, prefix=0, y_dtype=torch.float32)
    assert torch.count_nonzero(y).item() == 0
    bias = torch.randn(m.rows, device="cuda")
    y = pm.gemv(x, prefix=0, bias=bias, y_dtype=torch.float32)
    assert torch.equal(y, bias.expand(3, -1))


@pytest.mark.parametrize("streamk", [False, True])
def test_split_rows_deterministic(streamk):
    """Split tile rows (stream-K kernel) and warp-split row blocks (row-block kernel) give
    identical bytes run to run."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(11)
    m = random_matrix(rng, 1000, 3000)
    pm = plane_matrix(m)
    x = torch.from_numpy(rng.standard_normal((4, m.cols)).astype(np.float16)).cuda()
    ws = pm.workspace(4)
    fl = hqb.FLAG_STREAMK if streamk else hqb.FLAG_ROWBLOCK
    outs = [pm.gemv(x, prefix=p, y_dtype=torch.float32, workspace=ws, flags=fl).cpu().numpy() for p in (1, 3, 4, 3)]
    assert outs[1].tobytes() == outs[3].tobytes()
    e64 = _fp64_reference(m, x.float().cpu().numpy(), 4)
    assert_close(outs[2], e64, 2e-4, 2e-4, "split rows p4")
    assert ws.error_flags() == 0


@pytest.mark.parametrize("rows,cols", [(16, 300), (1000, 3000), (1024, 4096), (200, 11008), (7168, 256)])
def test_row_block_kernel_matches_stream_k(rows, cols):
    """The row-block kernel (no tile row split between CTAs; the warps' parts of a row
    block summed in shared memory in warp order) against the FP64 reference and the
    stream-K kernel at every depth, batch 1/2/3/8, FP16 and FP32 activations, with bias
    (FP16 x at batch <= 2: both kernels on int8 activation limbs, also checked against
    their FP16-fragment forms).
    The shapes cover fewer (tile, stage) units than warps (16x300 at depth 1), a single
    CTA wave, 86 tile columns, and CTAs that take several row blocks in turn (7168x256).
    Repeated calls are bit-identical and leave no device error."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(rows * 3 + cols)
    m = random_matrix(rng, rows, cols)
    pm = plane_matrix(m)
    ws = pm.workspace(8, hqb.F32)  # large enough for FP16 activations too
    bias = rng.standard_normal(rows).astype(np.float32)
    bt = torch.from_numpy(bias).cuda()
    w64 = {p: orc.dequantize_prefix_np(m, p).astype(np.float64) for p in (1, 2, 3, 4)}
    for batch in (1, 2, 3, 8):
        x = rng.standard_normal((batch, cols)).astype(np.float16).astype(np.float32)
        for xdt in (torch.float16, torch.float32):
            xt = torch.from_numpy(x).cuda().to(xdt)
            for p in (1, 2, 3, 4):
                rb = hqb.FLAG_ROWBLOCK
                a = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float32, workspace=ws, flags=rb)
                a2 = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float32, workspace=ws, flags=rb | hqb.FLAG_PDL)
                b = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float32, workspace=ws, flags=hqb.FLAG_STREAMK)
                if xdt == torch.float16 and batch <= 2:  # int8-limb forms against the FP16-fragment forms
                    c = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float32, workspace=ws, flags=rb | hqb.FLAG_F16MMA)
                    assert rel_l2(a.cpu().numpy(), c.cpu().numpy()) <= 2e-5, f"row-block int8 vs FP16 b{batch} p{p}"
                torch.cuda.synchronize()
                assert torch.equal(a, a2), (batch, xdt, p)
                e64 = x.astype(np.float64) @ w64[p].T + bias[None, :]
                an = a.cpu().numpy()
                assert_close(an, e64, 2e-4, 2e-4, f"row-block b{batch} {xdt} p{p}")
                assert rel_l2(an, e64) <= 1e-3
                assert_close(an, b.cpu().numpy(), 2e-4, 2e-4, f"row-block vs stream-K b{batch} {xdt} p{p}")
    assert ws.error_flags() == 0


def test_workspace_shared_across_kernels():
    """One workspace through every kernel in turn: the stream-K kernel's flagged split-row
    words, the fix-up kernel's and the tcgen05 kernel's partial sums all leave the
    partials region zero, so each later call is right and the stream-K results repeat
    bit for bit."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(31)
    m = random_matrix(rng, 1000, 3000)
    pm = plane_matrix(m)
    depth = torch.from_numpy(rng.integers(1, 5, size=(pm.grid_rows, pm.grid_cols)).astype(np.uint8)).cuda()
    plan = hqb.DepthPlan(depth, 4)
    ws = pm.workspace(4)
    w64 = {p: orc.dequantize_prefix_np(m, p).astype(np.float64) for p in (2, 3)}
    for batch in (1, 4):
        x = rng.standard_normal((batch, m.cols)).astype(np.float16).astype(np.float32)
        xt = torch.from_numpy(x).cuda().half()
        ref = {p: x.astype(np.float64) @ w64[p].T for p in (2, 3)}
        sk = []
        for fl, p in ((hqb.FLAG_STREAMK, 3), (hqb.FLAG_RING, 3), (hqb.FLAG_STREAMK, 3), (hqb.FLAG_TCGEN05, 2),
                      (hqb.FLAG_STREAMK, 3), (None, None), (hqb.FLAG_STREAMK, 3), (hqb.FLAG_ROWBLOCK, 2),
                      (hqb.FLAG_STREAMK, 3)):
            if fl is None:  # per-tile depth: the depth-map kernel and the fix-up kernel
                pm.gemv(xt, depth=plan, y_dtype=torch.float32, workspace=ws)
                continue
            y = pm.gemv(xt, prefix=p, y_dtype=torch.float32, workspace=ws, flags=fl).cpu().numpy()
            assert_close(y, ref[p], 2e-4, 2e-4, f"b{batch} flags {fl}")
            if fl == hqb.FLAG_STREAMK:
                sk.append(y)
        assert all(a.tobytes() == sk[0].tobytes() for a in sk)
    assert ws.error_flags() == 0


def test_mixed_depth_against_oracle():
    rng = np.random.default_rng(7)
    m = random_matrix(rng, 520, 700)
    pm = plane_matrix(m)
    gr, gc = m.grid
    depth = rng.integers(1, 5, size=(gr, gc), dtype=np.uint8)
    import harpq_b200 as hqb

    plan = hqb.DepthPlan(torch.from_numpy(depth).cuda(), pm.stage_count)
    assert int(plan.flags.item()) == 0
    assert plan.plan.cpu().numpy()[-1] == int(depth.sum())
    w = pm.decode(depth=plan.depth).cpu().numpy()
    assert w.tobytes() == orc.dequantize_mixed(m, depth).tobytes()
    for batch in (1, 3, 12):
        x = rng.standard_normal((batch, m.cols)).astype(np.float16).astype(np.float32)
        bias = rng.standard_normal(m.rows).astype(np.float32)
        y = pm.gemv(torch.from_numpy(x).cuda().half(), depth=plan, bias=torch.from_numpy(bias).cuda(),
                    y_dtype=torch.float32).cpu().numpy()
        scalar = orc.linear_mixed(m, x, depth, bias)
        assert_close(y, scalar, 2e-4, 2e-4, f"mixed b{batch}")
    # a uniform depth map computes the uniform prefix (different kernels and FP32
    # summation orders: equal within the FP32 contract)
    for p in (1, 4):
        u = hqb.DepthPlan(torch.full((gr, gc), p, dtype=torch.uint8, device="cuda"), 4)
        x = torch.randn(2, m.cols, device="cuda").half()
        a = pm.gemv(x, depth=u, y_dtype=torch.float32).cpu().numpy()
        b = pm.gemv(x, prefix=p, y_dtype=torch.float32).cpu().numpy()
        assert_close(a, b, 2e-4, 2e-4, f"depth map of {p} vs prefix {p}")


def test_depth_plan_flags_bad_entries():
    import harpq_b200 as hqb

    depth = torch.tensor([[0, 2], [5, 1]], dtype=torch.uint8, device="cuda")
    plan = hqb.DepthPlan(depth, 4)
    assert int(plan.flags.item()) & hqb.DEVERR_DEPTH
    assert plan.plan.cpu().tolist() == [0, 3, 8]  # 0 -> 1 and 5 -> 4


def test_repack_flags_bad_scales():
    import harpq_b200 as hqb

    rng = np.random.default_rng(3)
    m = random_matrix(rng, 128, 128, stages=1)
    codes = torch.from_numpy(m.codes[0]).cuda()
    bits = torch.from_numpy(m.scales[0].astype(np.float16).view(np.int16)).cuda()
    bits[5] = 0x7E00  # NaN
    pm = hqb.PlaneMatrix(128, 128)
    pm.add_stage(codes, bits)
    assert int(pm.repack_flags.item()) & hqb.DEVERR_SCALE


def test_progressive_stage_append_matches_full_build():
    """Stages repacked one at a time (residency grows) give the same results."""
    rng = np.random.default_rng(21)
    m = random_matrix(rng, 256, 256)
    full = plane_matrix(m)
    import harpq_b200 as hqb
    from conftest import device_stages

    codes, bits, _ = device_stages(m)
    grow = hqb.PlaneMatrix(m.rows, m.cols)
    x = torch.randn(1, m.cols, device="cuda").half()
    for s in range(4):
        grow.add_stage(codes[s], bits[s])
        assert torch.equal(grow.gemv(x, prefix=s + 1, y_dtype=torch.float32),
                           full.gemv(x, prefix=s + 1, y_dtype=torch.float32))


@pytest.mark.parametrize("rows,cols", [(1, 1), (129, 127), (4096, 128), (128, 4224)])
def test_edge_shapes(rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    m = random_matrix(rng, rows, cols)
    pm = plane_matrix(m)
    assert pm.decode(4).cpu().numpy().tobytes() == orc.dequantize_prefix_np(m, 4).tobytes()
    x = rng.standard_normal((2, cols)).astype(np.float16).astype(np.float32)
    y = pm.gemv(torch.from_numpy(x).cuda().half(), prefix=4, y_dtype=torch.float32).cpu().numpy()
    assert_close(y, _fp64_reference(m, x, 4), 2e-4, 2e-4, f"{rows}x{cols}")


def test_simt_comparison_kernel_matches():
    import harpq_b200 as hqb

    rng = np.random.default_rng(5)
    m = random_matrix(rng, 384, 640)
    pm = plane_matrix(m)
    for batch in (1, 4, 8):
        x = rng.standard_normal((batch, m.cols)).astype(np.float16).astype(np.float32)
        y = pm.gemv(torch.from_numpy(x).cuda().half(), prefix=3, y_dtype=torch.float32,
                    flags=hqb.FLAG_SIMT).cpu().numpy()
        assert_close(y, _fp64_reference(m, x, 3), 2e-4, 2e-4, f"simt b{batch}")


def test_prepared_activations_shared_across_matrices():
    import harpq_b200 as hqb

    rng = np.random.default_rng(9)
    a = plane_matrix(random_matrix(rng, 256, 512))
    b = plane_matrix(random_matrix(rng, 640, 512))
    x = torch.randn(3, 512, device="cuda").half()
    xf = hqb.prepare_x(x)
    for pm in (a, b):
        ya = pm.gemv(x, prefix=2, y_dtype=torch.float32, x_prepared=xf)
        yb = pm.gemv(x, prefix=2, y_dtype=torch.float32)
        assert torch.equal(ya, yb)
        # the tcgen05 comparison kernel: equal within the FP32 contract (another summation order)
        yc = pm.gemv(x, prefix=2, y_dtype=torch.float32, flags=hqb.FLAG_TCGEN05)
        assert_close(yc.cpu().numpy(), yb.cpu().numpy(), 2e-4, 2e-4, "tcgen05 vs mma.sync kernel")
    # PDL launch flag gives the same result
    y1 = a.gemv(x, prefix=3, y_dtype=torch.float32, x_prepared=xf, flags=hqb.FLAG_PDL)
    y2 = a.gemv(x, prefix=3, y_dtype=torch.float32, x_prepared=xf)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


def test_invalid_arguments_rejected_without_launch():
    import harpq_b200 as hqb

    rng = np.random.default_rng(2)
    pm = plane_matrix(random_matrix(rng, 128, 128))
    x = torch.randn(1, 128, device="cuda").half()
    with pytest.raises(hqb.HQBError) as e:
        pm.gemv(x, prefix=5)
    assert e.value.status == 1
    with pytest.raises(hqb.HQBError):
        pm.gemv(torch.randn(17, 128, device="cuda").half(), prefix=1)
    with pytest.raises(hqb.HQBError):
        pm.gemv(x, prefix=1, flags=hqb.FLAG_SIMT, y_dtype=torch.float32, workspace=hqb.Workspace(256))
    with pytest.raises(hqb.HQBError) as e:
        pm.gemv(x, prefix=1, flags=hqb.FLAG_STREAMK | hqb.FLAG_ROWBLOCK)
    assert e.value.status == 1


@pytest.mark.parametrize("rows,cols", [(128, 128), (256, 1024), (1024, 512), (2048, 2048), (4096, 4096),
                                       (384, 8192)])
def test_pdl_launch_matches_plain_launch(rows, cols):
    """Programmatic-dependent launches (activations fetched after the wait) across
    schedules of every length relative to the ring give the same bytes as plain
    launches and leave no device error."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(rows + cols)
    pm = plane_matrix(random_matrix(rng, rows, cols))
    x = torch.randn(2, cols, device="cuda").half()
    xf = hqb.prepare_x(x)
    ws = pm.workspace(2)
    for p in (1, 2, 3, 4):
        a = pm.gemv(x, prefix=p, y_dtype=torch.float32, x_prepared=xf, workspace=ws, flags=hqb.FLAG_PDL)
        b = pm.gemv(x, prefix=p, y_dtype=torch.float32, x_prepared=xf, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(a, b), f"p{p}"
    assert ws.error_flags() == 0


def test_row_stacked_matrices_match_members():
    """A row-stack of matrices that share their input (fused q|k|v style) computes every
    member's GEMV in one launch; each member's slice equals its own GEMV, and padding
    rows of a member inside the stack decode to zero."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(77)
    members = [random_matrix(rng, r, 300, stages=3) for r in (256, 200, 130)]
    pms = [plane_matrix(m) for m in members]
    stack = hqb.PlaneMatrix.stack(pms)
    assert stack.row_offsets == [0, 256, 512] and stack.rows == 512 + 130
    x = torch.from_numpy(rng.standard_normal((2, 300)).astype(np.float32)).cuda().half()
    for p in (1, 3):
        ys = stack.split_rows(stack.gemv(x, prefix=p, y_dtype=torch.float32))
        for pm, m, got in zip(pms, members, ys):
            want = pm.gemv(x, prefix=p, y_dtype=torch.float32)
            assert_close(got.cpu().numpy(), want.cpu().numpy(), 2e-4, 2e-4, f"stacked member p{p}")
            assert got.shape[-1] == m.rows
    w = stack.decode(3).cpu().numpy()
    assert w[:256].tobytes() == orc.dequantize_prefix(members[0], 3).tobytes()
    assert w[256:456].tobytes() == orc.dequantize_prefix(members[1], 3).tobytes()
    assert np.all(w[456:512] == 0.0)
    assert w[512:].tobytes() == orc.dequantize_prefix(members[2], 3).tobytes()


@pytest.mark.parametrize("cols,xdt,misalign", [(300, torch.float16, False), (300, torch.float32, False),
                                               (1000, torch.float16, False), (1000, torch.float16, True),
                                               (1027, torch.float32, True), (4096, torch.float32, False)])
def test_in_kernel_activation_prep_matches_prepared(cols, xdt, misalign):
    """Raw activations prepared inside the GEMV (vector or scalar staging) give the
    bit-identical result of a separately prepared buffer."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(cols)
    pm = plane_matrix(random_matrix(rng, 384, cols))
    for batch in (1, 5, 12):
        off = 1 if misalign else 0
        buf = torch.randn(batch * cols + off, device="cuda").to(xdt)
        buf[off:off + cols] *= 40.0  # a wide dynamic range inside tiles
        x = buf[off:].view(batch, cols)
        xf = hqb.prepare_x(x)
        for p in (1, 4):
            ya = pm.gemv(x, prefix=p, y_dtype=torch.float32, x_prepared=xf)
            # raw FP16 x at batch <= 2 defaults to int8 limbs: pin the FP16-fragment form
            yb = pm.gemv(x, prefix=p, y_dtype=torch.float32, flags=hqb.FLAG_F16MMA)
            assert torch.equal(ya, yb), (batch, p)


@pytest.mark.parametrize("batch", [1, 3, 8])
def test_tcgen05_kernel_ring_wrap_and_pdl(batch):
    """The tcgen05 comparison kernel (HQB_FLAG_TCGEN05: raw FP16 activations, batch <= 8)
    on a layer whose CTAs hold more tiles than the shared-memory ring has slots at
    prefixes 2-4: against the FP64 materialize-then-matvec result, against the default
    mma.sync kernel, and bit-identical between plain and programmatic-dependent launches."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(4242 + batch)
    m = random_matrix(rng, 4096, 8192)
    pm = plane_matrix(m)
    x = (rng.standard_normal((batch, m.cols)) * 2.0).astype(np.float16).astype(np.float32)
    xt = torch.from_numpy(x).cuda().half()
    ws = pm.workspace(batch)
    for p in (1, 2, 4):
        tc = hqb.FLAG_TCGEN05
        y = pm.gemv(xt, prefix=p, y_dtype=torch.float32, workspace=ws, flags=tc).cpu().numpy()
        e64 = _fp64_reference(m, x, p)
        assert rel_l2(y, e64) <= 1e-3
        assert_close(y, e64, 2e-4, 2e-4, f"tcgen05 p{p}")
        y_mma = pm.gemv(xt, prefix=p, y_dtype=torch.float32, workspace=ws).cpu().numpy()
        assert_close(y, y_mma, 2e-4, 2e-4, f"tcgen05 vs mma.sync p{p}")
        y_pdl = pm.gemv(xt, prefix=p, y_dtype=torch.float32, workspace=ws, flags=tc | hqb.FLAG_PDL)
        torch.cuda.synchronize()
        assert np.array_equal(y_pdl.cpu().numpy(), y), f"PDL p{p}"
    assert ws.error_flags() == 0


# ---- stream-K kernel on int8 activation limbs (FP16 x, batch <= 2) -------------------

def _limb_case(rows, cols, batch, seed, outliers):
    rng = np.random.default_rng(seed)
    m = random_matrix(rng, rows, cols)
    x = (rng.standard_normal((batch, cols)) * 2).astype(np.float16)
    if outliers:
        x[:, ::97] *= 20  # outlier channels (x20, as the calibration activations of the configs)
    bias = rng.standard_normal(rows).astype(np.float32)
    return m, x, bias


@pytest.mark.parametrize("rows,cols", [(300, 520), (1000, 3000), (4096, 4096), (200, 11008), (65536, 256)])
@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("outliers", [False, True])
def test_int8_limb_kernel_against_oracle(rows, cols, batch, outliers):
    """Every prefix, FP32 and FP16 outputs, against the scalar-order oracle (plain x) or
    the FP64 materialize-then-matvec (x with outlier channels, where the oracle's own FP32
    running sum drifts by more than the contract), and rel-L2 against FP64 always; the
    65536x256 case has CTAs whose tiles wrap around the two tile columns more than once."""
    import harpq_b200 as hqb

    m, x, bias = _limb_case(rows, cols, batch, rows + cols + batch, outliers)
    pm = plane_matrix(m)
    xt = torch.from_numpy(x).cuda()
    xf = x.astype(np.float32)
    bt = torch.from_numpy(bias).cuda()
    ws = pm.workspace(batch)
    fl = hqb.FLAG_STREAMK
    assert pm.uses_int8_limbs(batch, hqb.F16, 1, flags=fl)
    for p in (1, 2, 3, 4):
        y = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float32, workspace=ws, flags=fl).cpu().numpy()
        e64 = _fp64_reference(m, xf, p, bias)
        want = e64 if outliers else orc.linear_reference(m, xf, p, bias)
        assert_close(y, want, 2e-4, 2e-4, f"{rows}x{cols} b{batch} p{p}")
        assert rel_l2(y, e64) <= 2e-5, f"{rows}x{cols} b{batch} p{p} rel-L2 {rel_l2(y, e64):.2e}"
        y16 = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float16, workspace=ws, flags=fl).float().cpu().numpy()
        assert_close(y16, e64, 2e-4, FP16_RTOL, f"{rows}x{cols} b{batch} p{p} f16")
        # The FP16-fragment form removes the code offset (+2) after FP32 accumulation, so
        # near-zero outputs next to outlier channels carry cancellation error there; the
        # int8 form accumulates exactly.  Compare the two as vectors.
        y_ref16 = pm.gemv(xt, prefix=p, bias=bt, y_dtype=torch.float32, workspace=ws,
                          flags=fl | hqb.FLAG_F16MMA).cpu().numpy()
        assert rel_l2(y, y_ref16) <= 1e-4, f"{rows}x{cols} b{batch} p{p} vs FP16-fragment kernel"
        assert rel_l2(y, e64) <= rel_l2(y_ref16, e64) + 1e-7
    assert ws.error_flags() == 0


def test_int8_limb_kernel_repeatable_and_prepared_launch():
    """A layer large enough that one limb-preparation launch serves every CTA (more than
    24 tiles per CTA on average): bit-identical outputs call to call, FP64 parity through
    the bit-exact device decode."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(21)
    rows, cols = 16384, 8192
    m = random_matrix(rng, rows, cols, stages=2)
    pm = plane_matrix(m)
    x = torch.from_numpy((rng.standard_normal((1, cols)) * 3).astype(np.float16)).cuda()
    ws = pm.workspace(1)
    assert pm.uses_int8_limbs(1, hqb.F16, 2)
    assert pm.gemv_launches(1, hqb.F16, 2) == 2  # limb preparation + GEMV
    a = pm.gemv(x, prefix=2, y_dtype=torch.float32, workspace=ws)
    b = pm.gemv(x, prefix=2, y_dtype=torch.float32, workspace=ws)
    assert torch.equal(a, b)
    e64 = (x.double() @ pm.decode(2).double().T).cpu().numpy()
    assert_close(a.cpu().numpy(), e64, 2e-4, 2e-4, "16384x8192 p2")
    assert rel_l2(a.cpu().numpy(), e64) <= 2e-5
    assert ws.error_flags() == 0


def test_int8_limb_kernel_zero_and_extreme_activations():
    """All-zero tiles, a tile of FP16 subnormals and a tile reaching the FP16 maximum in
    one activation row (each x keeps at least 24 bits relative to its tile's largest |x|)."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(33)
    m = random_matrix(rng, 1024, 1024)
    pm = plane_matrix(m)
    x = np.zeros((2, 1024), np.float16)
    x[0, 128:256] = rng.standard_normal(128).astype(np.float16) * np.float16(2.0 ** -20)  # subnormals
    x[0, 256:384] = (rng.standard_normal(128) * 8192).astype(np.float16)
    x[0, 300] = np.float16(65504.0)
    x[1, 512:] = rng.standard_normal(512).astype(np.float16)
    xt = torch.from_numpy(x).cuda()
    xf = x.astype(np.float32)
    for batch in (1, 2):
        for p in (1, 4):
            y = pm.gemv(xt[:batch], prefix=p, y_dtype=torch.float32, flags=hqb.FLAG_STREAMK).cpu().numpy()
            e64 = _fp64_reference(m, xf[:batch], p)
            assert_close(y, orc.linear_reference(m, xf[:batch], p), 2e-4, 2e-4, f"b{batch} p{p}")
            assert rel_l2(y, e64) <= 2e-5


@pytest.mark.parametrize("rows,cols", [(300, 520), (11008, 4096), (200, 11008), (65536, 256)])
@pytest.mark.parametrize("batch", [1, 2])
def test_int8_limb_kernel_depth_map(rows, cols, batch):
    """A per-tile depth map on the int8 stream-K kernel (depth-4 form, each tile's stages
    cut by its depth, units split evenly over the CTAs): the scalar-order oracle for plain
    x, FP64 for x with outlier channels, repeatable bytes, no device error.  11008x4096 with
    the map of seed 7 is the mixed-depth configuration."""
    import harpq_b200 as hqb

    for outliers in (False, True):
        m, x, bias = _limb_case(rows, cols, batch, rows + 3 * cols + batch, outliers)
        pm = plane_matrix(m)
        gr, gc = m.grid
        depth = np.random.default_rng(7).integers(1, 5, size=(gr, gc)).astype(np.uint8)
        plan = hqb.DepthPlan(torch.from_numpy(depth).cuda(), pm.stage_count)
        assert pm.uses_int8_limbs(batch, hqb.F16, 0, mixed=True)
        xt = torch.from_numpy(x).cuda()
        xf = x.astype(np.float32)
        bt = torch.from_numpy(bias).cuda()
        ws = pm.workspace(batch)
        y = pm.gemv(xt, depth=plan, bias=bt, y_dtype=torch.float32, workspace=ws)
        y2 = pm.gemv(xt, depth=plan, bias=bt, y_dtype=torch.float32, workspace=ws)
        assert torch.equal(y, y2)
        y = y.cpu().numpy()
        e64 = _fp64_reference(m, xf, 4, bias, depth=depth)
        want = e64 if outliers else orc.linear_mixed(m, xf, depth, bias)
        assert_close(y, want, 2e-4, 2e-4, f"{rows}x{cols} b{batch} outliers={outliers}")
        assert rel_l2(y, e64) <= 2e-5
        assert ws.error_flags() == 0
    # uniform maps against the uniform prefix
    for p in (1, 3):
        u = hqb.DepthPlan(torch.full((gr, gc), p, dtype=torch.uint8, device="cuda"), 4)
        a = pm.gemv(xt, depth=u, y_dtype=torch.float32).cpu().numpy()
        b = pm.gemv(xt, prefix=p, y_dtype=torch.float32).cpu().numpy()
        assert rel_l2(a, b) <= 2e-5, f"depth map of {p} vs prefix {p}"


@pytest.mark.parametrize("batch", [1, 2])
def test_register_ring_int8_fp32_paths(batch):
    """The register-ring int8 kernels with FP32 activations (forced with HQB_FLAG_STREAMK;
    FP32 x takes the bulk kernel by default): the depth-map form, and a layer large enough
    for the standalone limb preparation launch (prep_limbs_kernel<float>, more than 24 tiles
    per CTA on average).  Against the scalar-order oracle / FP64."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(600 + batch)
    m = random_matrix(rng, 520, 700)
    pm = plane_matrix(m)
    gr, gc = m.grid
    depth = rng.integers(1, 5, size=(gr, gc)).astype(np.uint8)
    plan = hqb.DepthPlan(torch.from_numpy(depth).cuda(), 4)
    x = (rng.standard_normal((batch, m.cols)) * 3).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    fl = hqb.FLAG_STREAMK
    assert pm.uses_int8_limbs(batch, hqb.F32, 0, mixed=True, flags=fl)
    assert pm.gemv_kernel(batch, hqb.F32, 0, mixed=True, flags=fl) == "gemv_unit_kernel"
    y = pm.gemv(xt, depth=plan, y_dtype=torch.float32, flags=fl).cpu().numpy()
    assert_close(y, orc.linear_mixed(m, x, depth), 2e-4, 2e-4, f"depth map FP32 b{batch}")
    assert rel_l2(y, _fp64_reference(m, x, 4, depth=depth)) <= 2e-5
    # standalone FP32 limb preparation: 16384x8192
    rows, cols = 16384, 8192
    big = random_matrix(rng, rows, cols, stages=2)
    pb = plane_matrix(big)
    assert pb.gemv_launches(batch, hqb.F32, 2, flags=fl) == 2  # limb preparation + GEMV
    assert pb.uses_int8_limbs(batch, hqb.F32, 2, flags=fl)
    xb = torch.from_numpy((rng.standard_normal((batch, cols)) * 2).astype(np.float32)).cuda()
    yb = pb.gemv(xb, prefix=2, y_dtype=torch.float32, flags=fl)
    e64 = (xb.double() @ pb.decode(2).double().T).cpu().numpy()
    assert_close(yb.cpu().numpy(), e64, 2e-4, 2e-4, f"16384x8192 FP32 b{batch}")
    assert rel_l2(yb.cpu().numpy(), e64) <= 2e-5


@pytest.mark.parametrize("flags_name", ["STREAMK", "ROWBLOCK"])
def test_register_ring_int8_nonfinite_activations(flags_name):
    """FP16 activations holding Inf or NaN on the register-ring int8 kernels (the default for
    FP16 x at batch <= 2): every output of that batch row is NaN, the other row is exact."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(61)
    m = random_matrix(rng, 512, 640)
    pm = plane_matrix(m)
    fl = getattr(hqb, "FLAG_" + flags_name)
    for bad in (np.inf, -np.inf, np.nan):
        x = rng.standard_normal((2, m.cols)).astype(np.float16)
        x[0, 300] = bad
        y = pm.gemv(torch.from_numpy(x).cuda(), prefix=3, y_dtype=torch.float32, flags=fl).cpu().numpy()
        assert np.all(np.isnan(y[0])), bad
        assert_close(y[1], orc.linear_reference(m, x[1:].astype(np.float32), 3)[0], 2e-4, 2e-4, "clean row")
