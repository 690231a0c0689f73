"""PyTorch operator over the C ABI: ``torch.ops.harpq_b200.gemv``.

The reference lists a PyTorch custom-op wrapper over its native GEMV as planned work
(docs/RESEARCH_PLAN.md:106-107); it has no implementation to mirror.  This module
registers one through ``torch.library`` so the GEMV can sit inside PyTorch programs
(eager, CUDA graphs, and tracing through its fake kernel):

    import harpq_b200_ops  # registers the operator
    y = torch.ops.harpq_b200.gemv(x, planes, rows, cols, prefix, bias, torch.float16)

Arguments:
    x        [batch, cols] FP16 or FP32 CUDA tensor, batch 1..16
    planes   the matrix's stage planes in stage order (uint8 CUDA tensors of
             hqb_plane_bytes each, e.g. ``PlaneMatrix.planes``)
    rows, cols   the matrix's original shape
    prefix   stages to evaluate, 0..len(planes)
    bias     optional [rows] FP16 or FP32 CUDA tensor
    out_dtype    torch.float16 or torch.float32

It returns a new [batch, rows] tensor, computed by ``hqb_gemv`` on the current stream of
x's device: the same kernels and the same bits as ``PlaneMatrix.gemv``.  The operator has
only a CUDA kernel (a CPU tensor raises: there is no CPU fallback).  Its scratch workspace
is cached per (device, stream, matrix grid, batch, x dtype), so calls on different streams
never share one.
"""

import ctypes
from typing import List, Optional

import torch

import harpq_b200 as hqb

_WORKSPACES: dict = {}


def _plane_matrix(planes: List[torch.Tensor], rows: int, cols: int) -> "hqb.PlaneMatrixC":
    if not 1 <= len(planes) <= hqb.MAX_STAGES:
        raise ValueError(f"a plane matrix has 1..{hqb.MAX_STAGES} stage planes, got {len(planes)}")
    need = hqb.plane_bytes(hqb.geometry(rows, cols))
    for s, p in enumerate(planes):
        if p.dtype != torch.uint8 or not p.is_contiguous() or p.numel() < need:
            raise ValueError(f"plane {s} must be a contiguous uint8 tensor of at least {need} bytes")
    arr = (hqb.vp * hqb.MAX_STAGES)(*[p.data_ptr() for p in planes], *([None] * (hqb.MAX_STAGES - len(planes))))
    return hqb.PlaneMatrixC(rows, cols, -(-rows // hqb.TILE), -(-cols // hqb.TILE), len(planes), 0, arr)


def _workspace(m: "hqb.PlaneMatrixC", device: torch.device, stream: int, batch: int, x_dtype: int) -> "hqb.Workspace":
    key = (device.index, stream, m.grid_rows, m.grid_cols, m.stage_count, batch, x_dtype)
    ws = _WORKSPACES.get(key)
    if ws is None:
        nbytes = hqb.lib().hqb_workspace_bytes(ctypes.byref(m), batch, x_dtype, device.index)
        if nbytes == 0:
            raise ValueError("hqb_workspace_bytes rejected the matrix, batch or activation type")
        ws = _WORKSPACES[key] = hqb.Workspace(nbytes, device)
    return ws


@torch.library.custom_op("harpq_b200::gemv", mutates_args=(), device_types="cuda")
def gemv(x: torch.Tensor, planes: List[torch.Tensor], rows: int, cols: int, prefix: int,
         bias: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """y[b, r] = Σ_c x[b, c]·W_prefix[r, c] (+ bias[r]) over the plane matrix `planes`."""
    if x.dim() != 2 or x.shape[1] != cols:
        raise ValueError(f"x must be [batch, {cols}]")
    if out_dtype not in (torch.float16, torch.float32):
        raise ValueError("out_dtype must be torch.float16 or torch.float32")
    if any(p.device != x.device for p in planes) or (bias is not None and bias.device != x.device):
        raise ValueError("x, planes and bias must be on one device")
    x = x.contiguous()
    m = _plane_matrix(planes, rows, cols)
    xd = hqb._dtype_code(x)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    ws = _workspace(m, x.device, stream, x.shape[0], xd)
    y = torch.empty(x.shape[0], rows, dtype=out_dtype, device=x.device)
    if bias is not None:
        bias = bias.contiguous()
    status = hqb.lib().hqb_gemv(ctypes.byref(m), prefix, x.data_ptr(), xd, x.shape[0],
                                None if bias is None else bias.data_ptr(),
                                hqb.F32 if bias is None else hqb._dtype_code(bias), y.data_ptr(),
                                hqb._dtype_code(y), ws.ptr(), ws.nbytes, stream)
    hqb.check(status, "hqb_gemv")
    return y


@gemv.register_fake
def _gemv_fake(x, planes, rows, cols, prefix, bias=None, out_dtype=torch.float16):
    torch._check(x.dim() == 2 and x.shape[1] == cols, lambda: f"x must be [batch, {cols}]")
    return x.new_empty((x.shape[0], rows), dtype=out_dtype)
