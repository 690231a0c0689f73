"""Python binding of the C ABI in include/harpq_b200.h (ctypes over libharpq_b200.so).

Device memory is held in torch tensors (allocation, streams and events only); every
computation runs in the library's sm_100a kernels.  There is no fallback: importing
this module without the built library, or calling it without a CUDA device, raises.

    import harpq_b200 as hqb
    m = hqb.PlaneMatrix.from_stages(rows, cols, codes, fp16_scale_bits)  # repack on device
    y = m.gemv(x, prefix=2)                        # x: [batch, cols] FP16/FP32 CUDA tensor
    w = m.decode(prefix=2)                         # dense FP32, bit-exact decode
"""

from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Sequence

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libharpq_b200.so"

F32, F16 = 0, 1
FLAG_PDL, FLAG_SIMT, FLAG_RING, FLAG_TCGEN05, FLAG_STREAMK, FLAG_ROWBLOCK = 1, 2, 4, 8, 16, 32
FLAG_F16MMA = 64  # keep the GEMV kernels on FP16-fragment MMAs (no int8 activation limbs)
FLAG_BULK = 128  # bulk-copy kernel (batch <= 2, raw x): default for large layers, forced by this flag
RAW_GENERIC, RAW_REQUIRE_FAST = 1, 2  # hqb_raw_gemv_ex: per-element FMA kernel / int8 raw-layout kernel only
I8_LIMBS = 4
TILE = 128
RECORD_BYTES = 4352
MAX_STAGES = 4
MAX_BATCH = 16
DEVERR_SCALE, DEVERR_DEPTH, DEVERR_TIMEOUT, DEVERR_LAUNCH = 1, 2, 4, 8
HQB_OK, HQB_ERR_INVALID, HQB_ERR_UNSUPPORTED = 0, 1, 801
NOALLOC_SCRATCH_BYTES = 4 << 20
ERR_SCRATCH_LIMIT = 20001

u64, u32, i32, vp = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p


class Geometry(ctypes.Structure):
    _fields_ = [(n, u64) for n in ("original_rows", "original_columns", "padded_rows", "padded_columns",
                                   "tile_rows", "tile_columns", "group_size")]


class RawStage(ctypes.Structure):
    _fields_ = [("packed_codes", vp), ("packed_code_bytes", u64), ("scale_fp16_bits", vp), ("scale_count", u64)]


class CopyC(ctypes.Structure):
    _fields_ = [("dst", ctypes.c_void_p), ("src", ctypes.c_void_p), ("bytes", ctypes.c_uint64)]


class RawStageF32(ctypes.Structure):
    _fields_ = [("packed_codes", vp), ("packed_code_bytes", u64), ("scales", vp), ("scale_count", u64)]


class PlaneMatrixC(ctypes.Structure):
    _fields_ = [("rows", u64), ("cols", u64), ("grid_rows", u32), ("grid_cols", u32), ("stage_count", u32),
                ("reserved", u32), ("planes", vp * MAX_STAGES)]


class GemvCallC(ctypes.Structure):
    _fields_ = [("m", vp), ("prefix", u32), ("x_dtype", i32), ("depth", vp), ("depth_plan", vp), ("x", vp),
                ("batch", u32), ("x_prepared", i32), ("bias", vp), ("bias_dtype", i32), ("y_dtype", i32), ("y", vp),
                ("flags", u32), ("reserved", u32)]


class LaunchInfo(ctypes.Structure):
    _fields_ = [("launches", u32), ("int8_limbs", u32), ("grid", u32), ("block", u32), ("smem_bytes", u32),
                ("reserved", u32), ("kernel", ctypes.c_char * 40)]


MAX_PEERS = 8


class GatherC(ctypes.Structure):
    _fields_ = [("world", u32), ("rank", u32), ("slot_rows", u64), ("peer_y", vp * MAX_PEERS),
                ("peer_flags", vp * MAX_PEERS)]


EXPORTS = {
    "hqb_version": (i32, []),
    "hqb_status_string": (ctypes.c_char_p, [i32]),
    "hqb_plane_bytes": (u64, [ctypes.POINTER(Geometry)]),
    "hqb_repack_stage": (i32, [ctypes.POINTER(Geometry), ctypes.POINTER(RawStage), vp, vp, vp]),
    "hqb_xfrag_bytes": (u64, [u64, u32, i32]),
    "hqb_prepare_x": (i32, [vp, i32, u64, u32, vp, vp]),
    "hqb_workspace_bytes": (u64, [ctypes.POINTER(PlaneMatrixC), u32, i32, i32]),
    "hqb_workspace_init": (i32, [vp, u64, vp]),
    "hqb_workspace_error": (i32, [vp, ctypes.POINTER(i32), vp]),
    "hqb_depth_plan_bytes": (u64, [u32]),
    "hqb_depth_plan": (i32, [vp, u32, u32, u32, vp, vp, vp]),
    "hqb_gemv": (i32, [ctypes.POINTER(PlaneMatrixC), u32, vp, i32, u32, vp, i32, vp, i32, vp, u64, vp]),
    "hqb_gemv_mixed": (i32, [ctypes.POINTER(PlaneMatrixC), vp, vp, vp, i32, u32, vp, i32, vp, i32, vp, u64, vp]),
    "hqb_gemv_ex": (i32, [ctypes.POINTER(PlaneMatrixC), u32, vp, vp, vp, i32, u32, i32, vp, i32, vp, i32, vp, u64,
                          u32, vp]),
    "hqb_gemv_noalloc": (i32, [ctypes.POINTER(PlaneMatrixC), u32, vp, i32, u32, vp, i32, vp, i32, vp]),
    "hqb_gemv_batch": (i32, [ctypes.POINTER(GemvCallC), u32, vp, u64, vp]),
    "hqb_step_create": (i32, [ctypes.POINTER(GemvCallC), u32, vp, u64, ctypes.POINTER(vp)]),
    "hqb_step_create_grouped": (i32, [ctypes.POINTER(GemvCallC), u32, vp, u64, ctypes.POINTER(vp)]),
    "hqb_step_create_io": (i32, [ctypes.POINTER(GemvCallC), u32, vp, u64, ctypes.POINTER(CopyC), u32,
                                 ctypes.POINTER(CopyC), u32, i32, ctypes.POINTER(vp)]),
    "hqb_gemv_grouped": (i32, [ctypes.POINTER(GemvCallC), u32, vp, u64, vp]),
    "hqb_step_launch": (i32, [vp, vp]),
    "hqb_step_destroy": (i32, [vp]),
    "hqb_gemv_query": (i32, [ctypes.POINTER(PlaneMatrixC), u32, i32, i32, u32, i32, u32, ctypes.POINTER(LaunchInfo)]),
    "hqb_peer_alloc": (i32, [u64, ctypes.POINTER(vp), vp]),
    "hqb_peer_open": (i32, [vp, ctypes.POINTER(vp)]),
    "hqb_peer_close": (i32, [vp]),
    "hqb_peer_free": (i32, [vp]),
    "hqb_gemv_gather": (i32, [ctypes.POINTER(PlaneMatrixC), u32, vp, i32, u32, vp, i32, i32, ctypes.POINTER(GatherC),
                              vp, u64, u32, vp]),
    "hqb_gather_wait": (i32, [vp, u32, vp, vp, vp]),
    "hqb_gather_wait_ex": (i32, [vp, u32, vp, vp, u64, vp]),
    "hqb_gemv_noalloc_flags": (i32, [ctypes.POINTER(i32), i32, vp]),
    "hqb_gemv_noalloc_reset": (i32, [vp]),
    "hqb_gemv_noalloc_scratch": (i32, [ctypes.POINTER(vp)]),
    "hqb_decode_planes": (i32, [ctypes.POINTER(PlaneMatrixC), u32, vp, vp, u64, vp]),
    "hqb_prefill_workspace_bytes": (u64, [ctypes.POINTER(PlaneMatrixC)]),
    "hqb_prefill_gemm": (i32, [ctypes.POINTER(PlaneMatrixC), u32, vp, i32, u32, vp, i32, vp, i32, vp, u64, vp]),
    "hqb_raw_gemv": (i32, [ctypes.POINTER(Geometry), ctypes.POINTER(RawStage), u32, u32, vp, u64, vp, u64, vp, u64,
                           vp]),
    "hqb_raw_gemv_ex": (i32, [ctypes.POINTER(Geometry), ctypes.POINTER(RawStage), u32, u32, vp, u64, vp, u64, vp,
                              u64, u32, vp]),
    "hqb_raw_dequantize_stage": (i32, [ctypes.POINTER(Geometry), ctypes.POINTER(RawStageF32), u32, u32, vp, vp]),
    "hqb_raw_dequantize_prefix": (i32, [ctypes.POINTER(Geometry), ctypes.POINTER(RawStageF32), u32, u32, vp, vp]),
    "hqb_raw_linear_ordered": (i32, [ctypes.POINTER(Geometry), ctypes.POINTER(RawStageF32), u32, u32, vp, u64, vp,
                                     vp, vp]),
}

_lib = None


class HQBError(RuntimeError):
    def __init__(self, status: int, what: str):
        msg = lib().hqb_status_string(status).decode() if _lib is not None else str(status)
        super().__init__(f"{what}: status {status} ({msg})")
        self.status = status


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with __graft_entry__.build()")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in EXPORTS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        raise HQBError(status, what)


def _stream(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.float32:
        return F32
    raise TypeError(f"unsupported dtype {t.dtype}; use float16 or float32")


def geometry(rows: int, cols: int, tile: Sequence[int] = (TILE, TILE), group: int = TILE) -> Geometry:
    pr = -(-rows // tile[0]) * tile[0]
    pc = -(-cols // tile[1]) * tile[1]
    return Geometry(rows, cols, pr, pc, tile[0], tile[1], group)


def plane_bytes(g: Geometry) -> int:
    return lib().hqb_plane_bytes(ctypes.byref(g))


def xfrag_bytes(cols: int, batch: int, x_dtype: int) -> int:
    return lib().hqb_xfrag_bytes(cols, batch, x_dtype)


def prepare_x(x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Prepared activations for hqb_gemv_ex(x_prepared=1); shareable across matrices."""
    x = x.contiguous()
    batch, cols = x.shape
    n = xfrag_bytes(cols, batch, _dtype_code(x))
    if n == 0:
        raise ValueError("invalid activation shape/dtype")
    if out is None:
        out = torch.empty(n, dtype=torch.uint8, device=x.device)
    check(lib().hqb_prepare_x(_ptr(x), _dtype_code(x), cols, batch, _ptr(out), _stream(stream)), "hqb_prepare_x")
    return out


class Workspace:
    """Caller-owned scratch for GEMV launches (cleared once at allocation)."""

    def __init__(self, nbytes: int, device=None, stream=None):
        self.buf = torch.zeros(max(256, nbytes), dtype=torch.uint8, device=device or "cuda")
        self.nbytes = self.buf.numel()

    def ptr(self) -> int:
        return self.buf.data_ptr()

    def error_flags(self, stream=None) -> int:
        out = ctypes.c_int(0)
        check(lib().hqb_workspace_error(self.ptr(), ctypes.byref(out), _stream(stream)), "hqb_workspace_error")
        return out.value

    def reset(self, stream=None) -> None:
        check(lib().hqb_workspace_init(self.ptr(), self.nbytes, _stream(stream)), "hqb_workspace_init")


class DepthPlan:
    """Per-tile depth map (uint8 [grid_rows, grid_cols]) and its device schedule."""

    def __init__(self, depth: torch.Tensor, stage_count: int, stream=None):
        if depth.dtype != torch.uint8 or depth.dim() != 2:
            raise TypeError("depth must be a uint8 [grid_rows, grid_cols] tensor")
        self.depth = depth.contiguous()
        self.grid_rows, self.grid_cols = self.depth.shape
        self.plan = torch.empty(self.grid_rows + 1, dtype=torch.int32, device=depth.device)
        self.flags = torch.zeros(1, dtype=torch.int32, device=depth.device)
        check(lib().hqb_depth_plan(_ptr(self.depth), self.grid_rows, self.grid_cols, stage_count, _ptr(self.plan),
                                   _ptr(self.flags), _stream(stream)), "hqb_depth_plan")


class PlaneMatrix:
    """A device-resident progressive matrix in the plane layout (one buffer per stage)."""

    def __init__(self, rows: int, cols: int, device=None):
        self.rows, self.cols = rows, cols
        self.geom = geometry(rows, cols)
        self.grid_rows, self.grid_cols = -(-rows // TILE), -(-cols // TILE)
        self.device = torch.device(device or "cuda")
        self.planes: list[torch.Tensor] = []
        self.repack_flags = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._ws: dict = {}

    @property
    def stage_count(self) -> int:
        return len(self.planes)

    def add_stage(self, codes: torch.Tensor, fp16_scale_bits: torch.Tensor, stream=None) -> None:
        """Repack one newly resident stage (reference layout, on device) into a new plane."""
        if self.stage_count >= MAX_STAGES:
            raise ValueError("a progressive matrix holds at most four stages")
        codes = codes.contiguous()
        bits = fp16_scale_bits.contiguous()
        plane = torch.empty(plane_bytes(self.geom), dtype=torch.uint8, device=self.device)
        st = RawStage(codes.data_ptr(), codes.numel(), bits.data_ptr(), bits.numel())
        check(lib().hqb_repack_stage(ctypes.byref(self.geom), ctypes.byref(st), _ptr(plane), _ptr(self.repack_flags),
                                     _stream(stream)), "hqb_repack_stage")
        self.planes.append(plane)

    @classmethod
    def stack(cls, mats: Sequence["PlaneMatrix"]) -> "PlaneMatrix":
        """Row-stacked matrix of matrices with equal column counts.  Matrices that share
        their input (q|k|v, gate|up) then run as one GEMV launch.  Tile records are
        tile-row major, so stacking is concatenation of the plane buffers.  Member i's
        outputs are rows [row_offsets[i], row_offsets[i] + member_rows[i]) of the result
        (split_rows).  Offsets are multiples of 128: a member whose row count is not a
        multiple of 128 keeps its zero padding rows inside the stack.  The stack holds
        the stages that every member holds."""
        if not mats:
            raise ValueError("nothing to stack")
        cols = mats[0].cols
        if any(m.cols != cols for m in mats):
            raise ValueError("stacked matrices need equal column counts")
        offsets, r = [], 0
        for m in mats:
            offsets.append(r)
            r += m.grid_rows * TILE
        out = cls(offsets[-1] + mats[-1].rows, cols, device=mats[0].device)
        stages = min(m.stage_count for m in mats)
        out.planes = [torch.cat([m.planes[s] for m in mats]) for s in range(stages)]
        out.row_offsets = offsets
        out.member_rows = [m.rows for m in mats]
        return out

    def split_rows(self, y: torch.Tensor) -> list[torch.Tensor]:
        """Views of each member's outputs in a stacked matrix's result [..., rows]."""
        offsets = getattr(self, "row_offsets", [0])
        rows = getattr(self, "member_rows", [self.rows])
        return [y[..., o:o + n] for o, n in zip(offsets, rows)]

    @classmethod
    def from_stages(cls, rows: int, cols: int, codes: Sequence[torch.Tensor], fp16_scale_bits: Sequence[torch.Tensor],
                    stream=None) -> "PlaneMatrix":
        m = cls(rows, cols, device=codes[0].device)
        for c, s in zip(codes, fp16_scale_bits):
            m.add_stage(c, s, stream)
        return m

    def c_struct(self) -> PlaneMatrixC:
        """The C view of this matrix, built once per set of planes (kept while they are)."""
        key = tuple(p.data_ptr() for p in self.planes)
        cached = getattr(self, "_c", None)
        if cached is None or cached[0] != key:
            arr = (vp * MAX_STAGES)(*key, *([None] * (MAX_STAGES - len(key))))
            cached = (key, PlaneMatrixC(self.rows, self.cols, self.grid_rows, self.grid_cols, len(key), 0, arr))
            self._c = cached
        return cached[1]

    def workspace_bytes(self, batch: int, x_dtype: int = F16) -> int:
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        return lib().hqb_workspace_bytes(ctypes.byref(self.c_struct()), batch, x_dtype, dev)

    def workspace(self, batch: int, x_dtype: int = F16) -> Workspace:
        key = (batch, x_dtype)
        if key not in self._ws:
            self._ws[key] = Workspace(self.workspace_bytes(batch, x_dtype), self.device)
        return self._ws[key]

    def gemv(self, x: torch.Tensor, prefix: int | None = None, bias: torch.Tensor | None = None,
             out: torch.Tensor | None = None, y_dtype=torch.float16, depth: DepthPlan | None = None,
             workspace: Workspace | None = None, x_prepared: torch.Tensor | None = None, flags: int = 0,
             stream=None) -> torch.Tensor:
        """y[b, r] = Σ_c x[b, c]·W[r, c] (+ bias) at a uniform prefix or a depth map."""
        if x.dim() == 1:
            x = x.unsqueeze(0)
        x = x.contiguous()
        batch = x.shape[0]
        if x.shape[1] != self.cols:
            raise ValueError("x has the wrong number of columns")
        xd = _dtype_code(x)
        if out is None:
            out = torch.empty(batch, self.rows, dtype=y_dtype, device=self.device)
        ws = workspace or self.workspace(batch, xd)
        prefix = self.stage_count if prefix is None else prefix
        src = x if x_prepared is None else x_prepared
        status = lib().hqb_gemv_ex(ctypes.byref(self.c_struct()), prefix, None if depth is None else _ptr(depth.depth),
                                   None if depth is None else _ptr(depth.plan), _ptr(src), xd, batch,
                                   0 if x_prepared is None else 1, _ptr(bias),
                                   F32 if bias is None else _dtype_code(bias), _ptr(out), _dtype_code(out), ws.ptr(),
                                   ws.nbytes, flags, _stream(stream))
        check(status, "hqb_gemv_ex")
        return out

    def launch_info(self, batch: int, x_dtype: int, prefix: int, mixed: bool = False, flags: int = 0,
                    x_prepared: bool = False) -> LaunchInfo:
        """What one gemv() call enqueues on this device (the library's own choice, hqb_gemv_query)."""
        info = LaunchInfo()
        with torch.cuda.device(self.device):
            check(lib().hqb_gemv_query(ctypes.byref(self.c_struct()), prefix, 1 if mixed else 0, x_dtype, batch,
                                       1 if x_prepared else 0, flags, ctypes.byref(info)), "hqb_gemv_query")
        return info

    def uses_int8_limbs(self, batch: int, x_dtype: int, prefix: int, mixed: bool = False, flags: int = 0,
                        x_prepared: bool = False) -> bool:
        """Whether the GEMV kernel of one gemv() call multiplies int8 activation limbs."""
        return bool(self.launch_info(batch, x_dtype, prefix, mixed, flags, x_prepared).int8_limbs)

    def gemv_kernel(self, batch: int, x_dtype: int, prefix: int, mixed: bool = False, flags: int = 0,
                    x_prepared: bool = False) -> str:
        """Name of the GEMV kernel one gemv() call runs."""
        return self.launch_info(batch, x_dtype, prefix, mixed, flags, x_prepared).kernel.decode()

    def gemv_launches(self, batch: int, x_dtype: int, prefix: int, mixed: bool = False, flags: int = 0,
                      x_prepared: bool = False) -> int:
        """Kernels one gemv() call launches (activation preparation, GEMV, split-row fix-up)."""
        return int(self.launch_info(batch, x_dtype, prefix, mixed, flags, x_prepared).launches)

    def gemv_gather(self, x: torch.Tensor, gather: "Gather", prefix: int | None = None,
                    bias: torch.Tensor | None = None, workspace: Workspace | None = None, flags: int = 0,
                    stream=None) -> None:
        """This rank's row shard of the layer, its outputs written into every rank's
        gathered buffer (gather.out after gather.wait())."""
        if x.dim() == 1:
            x = x.unsqueeze(0)
        x = x.contiguous()
        batch = x.shape[0]
        xd = _dtype_code(x)
        ws = workspace or self.workspace(batch, xd)
        prefix = self.stage_count if prefix is None else prefix
        check(lib().hqb_gemv_gather(ctypes.byref(self.c_struct()), prefix, _ptr(x), xd, batch, _ptr(bias),
                                    F32 if bias is None else _dtype_code(bias),
                                    F16 if gather.y_dtype == torch.float16 else F32, ctypes.byref(gather.c),
                                    ws.ptr(), ws.nbytes, flags, _stream(stream)), "hqb_gemv_gather")

    def prefill(self, x: torch.Tensor, prefix: int, bias: torch.Tensor | None = None,
                y_dtype: torch.dtype = torch.float16, workspace: torch.Tensor | None = None,
                out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Large-batch product (hqb_prefill_gemm): FP16 x [batch][cols] -> y [batch][rows];
        the selected stages decoded into FP16 weights in `workspace` (a uint8 device tensor of
        prefill_workspace_bytes(), allocated here when not given), then a cuBLAS GEMM."""
        x = x if x.dim() == 2 else x.unsqueeze(0)
        if not x.is_contiguous():
            raise ValueError("x must be contiguous")
        y = out if out is not None else torch.empty(x.shape[0], self.rows, dtype=y_dtype, device=x.device)
        if workspace is None:
            workspace = torch.empty(self.prefill_workspace_bytes(), dtype=torch.uint8, device=x.device)
        check(lib().hqb_prefill_gemm(ctypes.byref(self.c_struct()), prefix, _ptr(x), _dtype_code(x), x.shape[0],
                                     _ptr(bias), F32 if bias is None else _dtype_code(bias), _ptr(y), _dtype_code(y),
                                     _ptr(workspace), workspace.numel(), _stream(stream)), "hqb_prefill_gemm")
        return y

    def prefill_workspace_bytes(self) -> int:
        return int(lib().hqb_prefill_workspace_bytes(ctypes.byref(self.c_struct())))

    def decode(self, prefix: int | None = None, depth: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        out = torch.empty(self.rows, self.cols, dtype=torch.float32, device=self.device)
        prefix = self.stage_count if prefix is None else prefix
        check(lib().hqb_decode_planes(ctypes.byref(self.c_struct()), prefix, _ptr(depth), _ptr(out), out.numel(),
                                      _stream(stream)), "hqb_decode_planes")
        return out


class Step:
    """A fixed list of GEMV calls (plane matrix, x, prefix, out, flags) on one stream with one
    workspace: the decode step's GEMVs for one host call.  graph=True (default) captures them
    once into a CUDA graph (hqb_step_create) and run() launches it; graph=False runs them
    through hqb_gemv_batch.  independent=True (no call reads another's output) runs them as
    one grouped kernel launch where they share its form (hqb_gemv_grouped).  Buffers are bound at construction; refill x and read out in
    place."""

    def __init__(self, calls, workspace: Workspace, graph: bool = True, independent: bool = False,
                 inputs=(), outputs=()):
        """inputs: (device tensor, pinned host tensor) copied host -> device before the GEMVs;
        outputs: (pinned host tensor, device tensor) copied device -> host after them; both
        are captured into the step's graph (hqb_step_create_io)."""
        self.calls = list(calls)
        self.handle = None
        self.independent = independent
        self.ws = workspace
        arr = (GemvCallC * len(self.calls))()
        self._keep = []
        for i, (pm, x, prefix, out, flags) in enumerate(self.calls):
            x = x if x.dim() == 2 else x.unsqueeze(0)
            if not x.is_contiguous() or not out.is_contiguous():
                raise ValueError("Step buffers must be contiguous")
            ms = pm.c_struct()
            self._keep.append(ms)
            arr[i] = GemvCallC(ctypes.addressof(ms), prefix, _dtype_code(x), None, None, x.data_ptr(), x.shape[0], 0,
                               None, F32, _dtype_code(out), out.data_ptr(), flags, 0)
        self.arr = arr
        if (inputs or outputs) and not graph:
            raise ValueError("input/output copies need graph=True")
        if graph:
            h = vp()
            if inputs or outputs:
                for dst, src in [*inputs, *outputs]:
                    if dst.numel() * dst.element_size() != src.numel() * src.element_size():
                        raise ValueError("copy sizes differ")
                    if not (dst.is_contiguous() and src.is_contiguous()):
                        raise ValueError("copy buffers must be contiguous")
                    host = src if src.device.type == "cpu" else dst
                    if not host.is_pinned():
                        raise ValueError("host buffers of a step must be pinned")
                self._io = [*inputs, *outputs]
                h2d = (CopyC * max(1, len(inputs)))(*[CopyC(d.data_ptr(), s_.data_ptr(), d.numel() * d.element_size())
                                                      for d, s_ in inputs])
                d2h = (CopyC * max(1, len(outputs)))(*[CopyC(d.data_ptr(), s_.data_ptr(), d.numel() * d.element_size())
                                                       for d, s_ in outputs])
                check(lib().hqb_step_create_io(arr, len(self.calls), self.ws.ptr(), self.ws.nbytes, h2d, len(inputs),
                                               d2h, len(outputs), 1 if independent else 0, ctypes.byref(h)),
                      "hqb_step_create_io")
            else:
                create = lib().hqb_step_create_grouped if independent else lib().hqb_step_create
                check(create(arr, len(self.calls), self.ws.ptr(), self.ws.nbytes, ctypes.byref(h)), "hqb_step_create")
            self.handle = h.value

    def run(self, stream=None) -> None:
        if self.handle is not None:
            check(lib().hqb_step_launch(self.handle, _stream(stream)), "hqb_step_launch")
        else:
            run = lib().hqb_gemv_grouped if self.independent else lib().hqb_gemv_batch
            check(run(self.arr, len(self.calls), self.ws.ptr(), self.ws.nbytes, _stream(stream)), "hqb_gemv_batch")

    def close(self) -> None:
        if self.handle is not None:
            lib().hqb_step_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RawMatrix:
    """Stages in the reference's own device layout (any tile geometry)."""

    def __init__(self, geom: Geometry, codes: Sequence[torch.Tensor], fp16_scale_bits: Sequence[torch.Tensor] = (),
                 scales_f32: Sequence[torch.Tensor] = ()):
        self.geom = geom
        self.codes = [c.contiguous() for c in codes]
        self.bits = [b.contiguous() for b in fp16_scale_bits]
        self.f32 = [s.contiguous() for s in scales_f32]

    def _stages(self):
        arr = (RawStage * MAX_STAGES)()
        for i, (c, b) in enumerate(zip(self.codes, self.bits)):
            arr[i] = RawStage(c.data_ptr(), c.numel(), b.data_ptr(), b.numel())
        return arr

    def _stages_f32(self):
        arr = (RawStageF32 * MAX_STAGES)()
        for i, (c, s) in enumerate(zip(self.codes, self.f32)):
            arr[i] = RawStageF32(c.data_ptr(), c.numel(), s.data_ptr(), s.numel())
        return arr

    def gemv(self, x: torch.Tensor, prefix: int, bias: torch.Tensor | None = None, stream=None,
             flags: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
        """LaunchProgressiveGemv semantics (hqb_raw_gemv_ex); flags RAW_GENERIC / RAW_REQUIRE_FAST."""
        y = out if out is not None else torch.empty(self.geom.original_rows, dtype=torch.float32, device=x.device)
        check(lib().hqb_raw_gemv_ex(ctypes.byref(self.geom), self._stages(), len(self.codes), prefix, _ptr(x),
                                    x.numel(), _ptr(bias), 0 if bias is None else bias.numel(), _ptr(y), y.numel(),
                                    flags, _stream(stream)), "hqb_raw_gemv_ex")
        return y

    def dequantize_prefix(self, prefix: int, stream=None) -> torch.Tensor:
        out = torch.empty(self.geom.original_rows, self.geom.original_columns, dtype=torch.float32,
                          device=self.codes[0].device)
        check(lib().hqb_raw_dequantize_prefix(ctypes.byref(self.geom), self._stages_f32(), len(self.codes), prefix,
                                              _ptr(out), _stream(stream)), "hqb_raw_dequantize_prefix")
        return out

    def dequantize_stage(self, stage: int, stream=None) -> torch.Tensor:
        out = torch.empty(self.geom.original_rows, self.geom.original_columns, dtype=torch.float32,
                          device=self.codes[0].device)
        check(lib().hqb_raw_dequantize_stage(ctypes.byref(self.geom), self._stages_f32(), len(self.codes), stage,
                                             _ptr(out), _stream(stream)), "hqb_raw_dequantize_stage")
        return out

    def linear_ordered(self, x: torch.Tensor, prefix: int, bias: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        x = x.contiguous().reshape(-1, self.geom.original_columns)
        y = torch.empty(x.shape[0], self.geom.original_rows, dtype=torch.float32, device=x.device)
        check(lib().hqb_raw_linear_ordered(ctypes.byref(self.geom), self._stages_f32(), len(self.codes), prefix,
                                           _ptr(x), x.shape[0], _ptr(bias), _ptr(y), _stream(stream)),
              "hqb_raw_linear_ordered")
        return y


# ---- output-row sharding across ranks --------------------------------------------------

def shard_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Tile-row aligned contiguous output rows of one rank: (first row, row count).

    Whole 128-row tiles are dealt out as evenly as possible, so every rank's shard is
    itself a valid plane matrix and the ranks' slices tile [0, rows) exactly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    tiles = -(-rows // TILE)
    t0, t1 = tiles * rank // world, tiles * (rank + 1) // world
    r0, r1 = t0 * TILE, min(t1 * TILE, rows)
    return r0, max(0, r1 - r0)


def shard_pad_rows(rows: int, world: int) -> int:
    """Per-rank slot size of the gathered output (the largest shard, whole tiles)."""
    return -(-(-(-rows // TILE)) // world) * TILE


def slice_stage_rows(codes, bits, cols: int, r0: int, nrows: int):
    """Row-shard one matrix's reference-layout stages (codes row-major, scales
    tile-row major): returns the (codes, fp16 bits) slices of rows [r0, r0+nrows)."""
    kpad = -(-cols // TILE) * TILE
    per_row = kpad // 4
    nt = -(-nrows // TILE)
    c = [x[r0 * per_row:(r0 + nt * TILE) * per_row] for x in codes]
    per_tile_row = (kpad // TILE) * TILE
    t0 = r0 // TILE
    b = [x[t0 * per_tile_row:(t0 + nt) * per_tile_row] for x in bits]
    return c, b


# ---------------------------------------------------------------------------------------
# output-row shards across the GPUs of one node: fused all-gather over peer memory

class _DeviceView:
    """Raw device memory seen as a torch tensor (CUDA array interface, no copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBuffer:
    """A device buffer of `nbytes` (zero-initialised) that every rank of a torch.distributed
    group maps: rank r's copy is peers[r] (peers[rank] is the local one).  Collective:
    every rank constructs it in the same order."""

    def __init__(self, nbytes: int, group=None):
        import torch.distributed as dist

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        local = vp()
        handle = ctypes.create_string_buffer(64)
        check(lib().hqb_peer_alloc(nbytes, ctypes.byref(local), handle), "hqb_peer_alloc")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        self.local = local.value
        self.peers = []
        self._opened = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.peers.append(self.local)
                continue
            ptr = vp()
            check(lib().hqb_peer_open(ctypes.create_string_buffer(h, 64), ctypes.byref(ptr)), "hqb_peer_open")
            self.peers.append(ptr.value)
            self._opened.append(ptr.value)
        self.nbytes = nbytes

    def close(self):
        for ptr in self._opened:
            lib().hqb_peer_close(ptr)
        self._opened = []
        if self.local:
            lib().hqb_peer_free(self.local)
            self.local = None


class Gather:
    """Gathered output of a row-sharded layer: [batch][world * slot_rows] of y_dtype on every
    rank, filled by PlaneMatrix.gemv_gather on all ranks; wait() orders later work in the
    stream after every rank's slice has arrived."""

    def __init__(self, slot_rows: int, batch: int = 1, y_dtype=torch.float16, group=None):
        self.slot_rows, self.batch = slot_rows, batch
        self.y_dtype = y_dtype
        esize = 2 if y_dtype == torch.float16 else 4
        self.ybuf = PeerBuffer(batch * slot_rows * _world(group) * esize, group)
        self.flags = PeerBuffer(4 * MAX_PEERS, group)
        self.epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.device_flags = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.world, self.rank = self.ybuf.world, self.ybuf.rank
        c = GatherC()
        c.world, c.rank, c.slot_rows = self.world, self.rank, slot_rows
        for r in range(self.world):
            c.peer_y[r] = self.ybuf.peers[r]
            c.peer_flags[r] = self.flags.peers[r]
        self.c = c
        self.out = torch.as_tensor(_DeviceView(self.ybuf.local, (batch, self.world * slot_rows),
                                               "<f2" if esize == 2 else "<f4"), device="cuda")

    def wait(self, stream=None):
        check(lib().hqb_gather_wait(self.flags.local, self.world, _ptr(self.epoch), _ptr(self.device_flags),
                                    _stream(stream)), "hqb_gather_wait")

    def close(self):
        self.ybuf.close()
        self.flags.close()


def _world(group=None) -> int:
    import torch.distributed as dist

    return dist.get_world_size(group)
