"""The torch.library operator torch.ops.harpq_b200.gemv, host side (no GPU needed).

Registration and schema, shape and dtype propagation through its fake kernel (meta
tensors, as tracing sees it), and that CPU tensors are refused (no CPU fallback).  The
operator's CUDA results are checked in tests/test_gpu_torch_op.py.
"""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

import harpq_b200 as hqb  # noqa: E402
import harpq_b200_ops  # noqa: E402,F401  (registers the operator)


def test_operator_is_registered_with_its_schema():
    op = torch.ops.harpq_b200.gemv.default
    schema = str(op._schema)
    assert schema.startswith("harpq_b200::gemv(Tensor x, Tensor[] planes, SymInt rows, SymInt cols, SymInt prefix")
    assert "Tensor? bias=None" in schema and "ScalarType out_dtype=" in schema and schema.endswith("-> Tensor")


@pytest.mark.parametrize("batch,out_dtype", [(1, torch.float16), (3, torch.float32), (16, torch.float16)])
def test_fake_kernel_shapes(batch, out_dtype):
    rows, cols = 300, 520
    nbytes = hqb.plane_bytes(hqb.geometry(rows, cols))
    x = torch.empty(batch, cols, dtype=torch.float16, device="meta")
    planes = [torch.empty(nbytes, dtype=torch.uint8, device="meta") for _ in range(3)]
    y = torch.ops.harpq_b200.gemv(x, planes, rows, cols, 2, None, out_dtype)
    assert y.shape == (batch, rows) and y.dtype == out_dtype and y.device.type == "meta"


def test_fake_kernel_checks_columns():
    x = torch.empty(2, 100, dtype=torch.float16, device="meta")
    planes = [torch.empty(16, dtype=torch.uint8, device="meta")]
    with pytest.raises(RuntimeError):
        torch.ops.harpq_b200.gemv(x, planes, 128, 128, 1, None, torch.float16)


def test_cpu_tensors_are_refused():
    x = torch.zeros(1, 128, dtype=torch.float16)
    planes = [torch.zeros(hqb.plane_bytes(hqb.geometry(128, 128)), dtype=torch.uint8)]
    with pytest.raises(NotImplementedError):
        torch.ops.harpq_b200.gemv(x, planes, 128, 128, 1, None, torch.float16)
