"""TEST INFRASTRUCTURE ONLY — ctypes binding of oracle/_ref/libharpq_ref.so.

That library is the reference's own native/src/stage_codec.cpp compiled in place
(see oracle/build.py).  Tests use it to pin the C restatement; bench.py's
reference arm times ``ProgressiveLinearReference`` through it, splitting a layer
into tile-row shards so every host core has work.
"""

from __future__ import annotations

import ctypes
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .oracle import REF_LIB_PATH, Matrix

_lib = None


class _Geo(ctypes.Structure):
    _fields_ = [("v", ctypes.c_uint64 * 7)]


class _Stage(ctypes.Structure):
    _fields_ = [("codes", ctypes.c_void_p), ("code_bytes", ctypes.c_uint64),
                ("scales", ctypes.c_void_p), ("scale_count", ctypes.c_uint64)]


def available() -> bool:
    return REF_LIB_PATH.exists()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(REF_LIB_PATH))
        vp, u64 = ctypes.c_void_p, ctypes.c_uint64
        L.hqr_crc32c.restype = ctypes.c_uint32
        L.hqr_crc32c.argtypes = [vp, u64, ctypes.c_uint32]
        L.hqr_decode_payload.restype = ctypes.c_int
        L.hqr_decode_payload.argtypes = [vp, u64, ctypes.c_uint16, vp, vp, vp]
        L.hqr_matrix_create.restype = vp
        L.hqr_matrix_create.argtypes = [ctypes.POINTER(_Geo), ctypes.POINTER(_Stage), ctypes.c_uint32]
        L.hqr_matrix_free.restype = None
        L.hqr_matrix_free.argtypes = [vp]
        L.hqr_dequantize_prefix.restype = ctypes.c_int
        L.hqr_dequantize_prefix.argtypes = [vp, ctypes.c_uint32, vp]
        L.hqr_linear_reference.restype = ctypes.c_int
        L.hqr_linear_reference.argtypes = [vp, ctypes.c_uint32, vp, u64, vp, vp]
        _lib = L
    return _lib


class RefMatrix:
    """A reference ``ProgressiveMatrix`` owned by the reference library."""

    def __init__(self, m: Matrix):
        self.rows, self.cols = m.rows, m.cols
        geo = _Geo()
        geo.v[:] = list(m.geometry)
        st = (_Stage * m.stage_count)()
        keep = []
        for i, (c, s) in enumerate(zip(m.codes, m.scales)):
            c = np.ascontiguousarray(c, np.uint8)
            s = np.ascontiguousarray(s, np.float32)
            keep += [c, s]
            st[i] = _Stage(c.ctypes.data, c.size, s.ctypes.data, s.size)
        self.handle = lib().hqr_matrix_create(ctypes.byref(geo), st, m.stage_count)
        if not self.handle:
            raise RuntimeError("reference ProgressiveMatrix construction failed")

    def __del__(self):
        if getattr(self, "handle", None):
            lib().hqr_matrix_free(self.handle)
            self.handle = None

    def dequantize_prefix(self, prefix: int) -> np.ndarray:
        out = np.zeros((self.rows, self.cols), np.float32)
        if lib().hqr_dequantize_prefix(self.handle, prefix, out.ctypes.data):
            raise ValueError("reference DequantizePrefix rejected the request")
        return out

    def linear(self, x: np.ndarray, prefix: int, bias: np.ndarray | None = None,
               out: np.ndarray | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.cols)
        if out is None:
            out = np.zeros((x.shape[0], self.rows), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        rc = lib().hqr_linear_reference(self.handle, prefix, x.ctypes.data, x.shape[0],
                                        None if b is None else b.ctypes.data, out.ctypes.data)
        if rc:
            raise ValueError("reference ProgressiveLinearReference rejected the request")
        return out


def row_shards(m: Matrix, shards: int) -> list[tuple[int, Matrix]]:
    """Split a matrix into tile-row aligned sub-matrices (row offset, Matrix).

    Codes are row-major over the padded matrix and scales are tile-row major, so
    a run of whole tile rows is a contiguous slice of both."""
    g = m.geometry
    rows, cols, rows_p, cols_p, tr, tc, grp = g
    grid_r = rows_p // tr
    shards = max(1, min(shards, grid_r))
    per_row_scales = (cols_p // tc) * tr * (tc // grp)
    out = []
    for k in range(shards):
        r0, r1 = grid_r * k // shards, grid_r * (k + 1) // shards
        if r1 == r0:
            continue
        row0 = r0 * tr
        nrows = min(r1 * tr, rows) - row0
        if nrows <= 0:
            continue
        geo = (nrows, cols, (r1 - r0) * tr, cols_p, tr, tc, grp)
        cb = (r1 - r0) * tr * cols_p // 4
        codes = [c[row0 * cols_p // 4: row0 * cols_p // 4 + cb] for c in m.codes]
        scales = [s[r0 * per_row_scales: r1 * per_row_scales] for s in m.scales]
        out.append((row0, Matrix(geo, codes, scales)))
    return out


class ShardedReference:
    """Reference ProgressiveLinearReference over tile-row shards on a thread pool."""

    def __init__(self, m: Matrix, threads: int):
        self.rows = m.rows
        self.threads = threads
        self.parts = [(row0, RefMatrix(sub)) for row0, sub in row_shards(m, threads)]
        self.pool = ThreadPoolExecutor(max_workers=threads)

    def linear(self, x: np.ndarray, prefix: int, bias: np.ndarray | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        out = np.zeros((x2.shape[0], self.rows), np.float32)

        def run(part):
            row0, rm = part
            b = None if bias is None else bias[row0: row0 + rm.rows]
            out[:, row0: row0 + rm.rows] = rm.linear(x2, prefix, b)

        list(self.pool.map(run, self.parts))
        return out

    def close(self):
        self.pool.shutdown()
