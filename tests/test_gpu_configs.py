"""GPU parity on the benchmarked configurations at their full sizes (random codes and
FP16-exact scales; the kernels do not depend on how the codes were fitted).

Each case runs the library's default kernel choice for the shape -- the kernels bench.py
times -- and checks it element by element against an FP64 materialize-then-matvec of the
bit-exact device decode (|a - e| <= 2e-4 + 2e-4*|e|, the reference's fused-GEMV tolerance,
native/tests/progressive_gemv_test.cu:36-37), and against the scalar-order
ProgressiveLinearReference restatement (oracle/harpq_oracle.c) by relative L2.

* config 3 (LLaMA-70B MLP): 28672x8192 at prefix 1 and 3, 8192x28672 at prefix 3;
* config 2 (LLaMA-7B block): the 4096x11008 down projection at every prefix, and the
  row-stacked q+k+v and gate+up launches exactly as bench.py builds them;
* config 5 (small batch, prefix 4): 4096x4096 and 11008x4096 at batch 4, 8 and 16.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from conftest import assert_close, plane_matrix, random_matrix, rel_l2  # noqa: E402
from oracle import oracle as orc  # noqa: E402


def _hqb():
    import harpq_b200 as hqb

    return hqb


def _e64(pm, prefix, x):
    """FP64 x @ W^T with W the bit-exact device decode (no FP64 copy of W on the host)."""
    w = pm.decode(prefix).double()
    return (torch.as_tensor(x, device="cuda").double() @ w.T).cpu().numpy()


@pytest.mark.parametrize("rows,cols,prefixes", [(28672, 8192, (1, 3)), (8192, 28672, (3,)), (4096, 11008, (1, 2, 3, 4))])
def test_full_size_batch_one(rows, cols, prefixes):
    hqb = _hqb()
    rng = np.random.default_rng(rows ^ cols)
    m = random_matrix(rng, rows, cols, stages=max(prefixes))
    pm = plane_matrix(m)
    x = rng.standard_normal((1, cols)).astype(np.float16)
    xt = torch.from_numpy(x).cuda()
    ws = pm.workspace(1)
    for p in prefixes:
        kernel = pm.gemv_kernel(1, hqb.F16, p)
        y = pm.gemv(xt, prefix=p, y_dtype=torch.float32, workspace=ws).cpu().numpy()
        y2 = pm.gemv(xt, prefix=p, y_dtype=torch.float32, workspace=ws).cpu().numpy()
        assert np.array_equal(y, y2), f"{kernel} p{p} not repeatable"
        e64 = _e64(pm, p, x.astype(np.float32))
        assert_close(y, e64, 2e-4, 2e-4, f"{rows}x{cols} p{p} ({kernel})")
        assert rel_l2(y, e64) <= 2e-5
        scalar = orc.linear_reference(m, x.astype(np.float32), p)
        assert rel_l2(y, scalar) <= 1e-5, f"{rows}x{cols} p{p} vs scalar-order oracle"
    assert ws.error_flags() == 0


@pytest.mark.parametrize("members,cols", [((4096, 4096, 4096), 4096), ((11008, 11008), 4096)])
def test_stacked_launch_as_benchmarked(members, cols):
    """q+k+v and gate+up: members row-stacked into one plane matrix (PlaneMatrix.stack) and
    run as one launch at prefix 2, batch 1, FP16 x and y, as in bench.py; every member's
    slice against its own FP64 result and its own launch."""
    hqb = _hqb()
    rng = np.random.default_rng(len(members) * 1000 + cols)
    mats = [random_matrix(rng, r, cols, stages=2) for r in members]
    pms = [plane_matrix(m) for m in mats]
    stack = hqb.PlaneMatrix.stack(pms)
    x = rng.standard_normal((1, cols)).astype(np.float16)
    xt = torch.from_numpy(x).cuda()
    ys = stack.split_rows(stack.gemv(xt, prefix=2, y_dtype=torch.float16, flags=hqb.FLAG_PDL))
    torch.cuda.synchronize()
    for pm, got in zip(pms, ys):
        e64 = _e64(pm, 2, x.astype(np.float32))
        assert_close(got.float().cpu().numpy(), e64, 2e-4, 2.0 ** -10, "stacked member (FP16 y)")
        alone = pm.gemv(xt, prefix=2, y_dtype=torch.float32).cpu().numpy()
        assert_close(got.float().cpu().numpy(), alone, 2e-4, 2.0 ** -10, "stacked vs alone")


@pytest.mark.parametrize("rows", [4096, 11008])
@pytest.mark.parametrize("batch", [4, 8, 16])
def test_small_batch_full_size(rows, batch):
    """Config 5 at full size: prefix 4, FP16 x, batch 4/8/16 on the FP16-fragment tensor-core
    kernel the benchmark times."""
    hqb = _hqb()
    rng = np.random.default_rng(rows + batch)
    m = random_matrix(rng, rows, 4096)
    pm = plane_matrix(m)
    x = rng.standard_normal((batch, 4096)).astype(np.float16)
    xt = torch.from_numpy(x).cuda()
    y = pm.gemv(xt, prefix=4, y_dtype=torch.float32).cpu().numpy()
    e64 = _e64(pm, 4, x.astype(np.float32))
    assert_close(y, e64, 2e-4, 2e-4, f"{rows}x4096 b{batch} ({pm.gemv_kernel(batch, hqb.F16, 4)})")
    assert rel_l2(y, e64) <= 1e-3
