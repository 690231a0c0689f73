"""torch.ops.harpq_b200.gemv on the B200: the same bits as PlaneMatrix.gemv (both reach
hqb_gemv_ex with no flags) and the oracle's result within the FP32 contract, for batch 1
and 3, FP16 and FP32 x, FP16 and FP32 outputs, every prefix, with and without bias; and
inside a captured CUDA graph."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from conftest import assert_close, plane_matrix, random_matrix  # noqa: E402
from oracle import oracle as orc  # noqa: E402


def test_operator_matches_plane_matrix_and_oracle():
    import harpq_b200_ops  # noqa: F401

    rng = np.random.default_rng(41)
    m = random_matrix(rng, 1000, 3000)
    pm = plane_matrix(m)
    bias = rng.standard_normal(m.rows).astype(np.float32)
    bt = torch.from_numpy(bias).cuda()
    for batch in (1, 3):
        x = rng.standard_normal((batch, m.cols)).astype(np.float16).astype(np.float32)
        for xdt in (torch.float16, torch.float32):
            xt = torch.from_numpy(x).cuda().to(xdt)
            for p in (0, 1, 2, 3, 4):
                for ydt in (torch.float16, torch.float32):
                    for b in (None, bt):
                        got = torch.ops.harpq_b200.gemv(xt, pm.planes, m.rows, m.cols, p, b, ydt)
                        want = pm.gemv(xt, prefix=p, bias=b, y_dtype=ydt)
                        assert torch.equal(got, want), (batch, xdt, p, ydt, b is None)
                e = orc.linear_reference(m, x, p, bias)
                got = torch.ops.harpq_b200.gemv(xt, pm.planes, m.rows, m.cols, p, bt, torch.float32)
                assert_close(got.cpu().numpy(), e, 2e-4, 2e-4, f"op b{batch} {xdt} p{p}")


def test_operator_in_a_cuda_graph():
    import harpq_b200_ops  # noqa: F401

    rng = np.random.default_rng(42)
    m = random_matrix(rng, 4096, 4096)
    pm = plane_matrix(m)
    x = torch.randn(1, m.cols, device="cuda").half()
    ref = torch.ops.harpq_b200.gemv(x, pm.planes, m.rows, m.cols, 2, None, torch.float16)  # warms the workspace
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        torch.ops.harpq_b200.gemv(x, pm.planes, m.rows, m.cols, 2, None, torch.float16)  # this stream's workspace
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g, stream=s):  # captured on s: the workspace warmed there
        y = torch.ops.harpq_b200.gemv(x, pm.planes, m.rows, m.cols, 2, None, torch.float16)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
