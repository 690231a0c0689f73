"""GPU: the prefill product (hqb_prefill_gemm) for batches far above the GEMV's 16.

The selected stages are decoded into FP16 weights and multiplied by cuBLAS (FP16 inputs,
FP32 accumulation).  Checks:
* the decoded FP16 weights are the FP32 DequantizePrefix restatement (plane decode, itself
  bit-exact against the oracle) rounded once to FP16, bit for bit;
* y against an FP64 product of the exact FP32 weights: rel-L2 <= 1e-3 (the north-star
  contract for the materialize-then-multiply result) and elementwise within the FP16 weight
  rounding (2^-11 relative per weight) and FP32 accumulation, bounded by
  2^-10 * sum|w||x| (+ 2^-10 |y| for FP16 outputs);
* prefix 0 writes bias or zeros; FP32 x is refused with HQB_ERR_UNSUPPORTED.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import harpq_b200 as hqb  # noqa: E402
from conftest import plane_matrix, random_matrix, rel_l2  # noqa: E402
from oracle import oracle as orc  # noqa: E402


@pytest.mark.parametrize("rows,cols,batch", [(300, 520, 32), (1000, 1100, 128), (4096, 4096, 256), (130, 4104, 64)])
def test_prefill_against_fp64(rows, cols, batch):
    rng = np.random.default_rng(rows + cols + batch)
    m = random_matrix(rng, rows, cols)
    pm = plane_matrix(m)
    x = rng.standard_normal((batch, cols)).astype(np.float16)
    xt = torch.from_numpy(x).cuda()
    bias = rng.standard_normal(rows).astype(np.float32)
    ws = torch.empty(pm.prefill_workspace_bytes(), dtype=torch.uint8, device="cuda")
    for p in (1, 2, 3, 4):
        w32 = orc.dequantize_prefix_np(m, p).astype(np.float64)
        for ydt, bt in ((torch.float32, torch.from_numpy(bias).cuda()), (torch.float16, None),
                        (torch.float32, torch.from_numpy(bias).half().cuda())):
            y = pm.prefill(xt, p, bias=bt, y_dtype=ydt, workspace=ws).float().cpu().numpy().astype(np.float64)
            b64 = 0.0 if bt is None else bt.float().cpu().numpy().astype(np.float64)
            e = x.astype(np.float64) @ w32.T + b64
            assert rel_l2(y, e) <= 1e-3, f"{rows}x{cols} b{batch} p{p} {ydt}"
            bound = 2.0 ** -10 * (np.abs(x.astype(np.float64)) @ np.abs(w32).T) + 1e-6
            if ydt == torch.float16:
                bound = bound + 2.0 ** -10 * np.abs(e)
            assert np.all(np.abs(y - e) <= bound), f"{rows}x{cols} b{batch} p{p} {ydt}"
        # the decoded weights: the FP32 prefix decode rounded once to FP16
        w16 = ws[: rows * cols * 2].view(torch.float16).view(rows, cols)
        assert torch.equal(w16, pm.decode(p).half()), f"decoded weights p{p}"


def test_prefill_prefix_zero_and_dtype_rules():
    rng = np.random.default_rng(3)
    m = random_matrix(rng, 256, 384)
    pm = plane_matrix(m)
    xt = torch.from_numpy(rng.standard_normal((40, 384)).astype(np.float16)).cuda()
    bt = torch.from_numpy(rng.standard_normal(256).astype(np.float32)).cuda()
    assert torch.equal(pm.prefill(xt, 0, bias=bt, y_dtype=torch.float32), bt.expand(40, -1))
    assert torch.count_nonzero(pm.prefill(xt, 0, y_dtype=torch.float32)).item() == 0
    with pytest.raises(hqb.HQBError) as ei:
        pm.prefill(xt.float(), 2)
    assert ei.value.status == hqb.HQB_ERR_UNSUPPORTED
    with pytest.raises(hqb.HQBError) as ei:
        pm.prefill(xt, 5)  # prefix beyond the stage count
    assert ei.value.status == hqb.HQB_ERR_INVALID
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(hqb.HQBError):
        pm.prefill(xt, 2, workspace=small)
