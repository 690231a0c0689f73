"""TEST INFRASTRUCTURE ONLY — Python binding of the CPU oracle (oracle/harpq_oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg
may import this module, and only to check or to time the reference arithmetic.
The product library (harp-q_b200/) never imports or calls it.

``dequantize_prefix_np`` is a vectorised NumPy form of the same arithmetic
(exact code*scale products, FP32 adds in stage order from 0.0f); the tests pin it
to the C oracle so it can check full-size layers quickly.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
LIB_PATH = ROOT / "liboracle.so"
REF_LIB_PATH = ROOT / "_ref" / "libharpq_ref.so"


class Geometry(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "original_rows", "original_columns", "padded_rows", "padded_columns",
        "tile_rows", "tile_columns", "group_size")]


class Stage(ctypes.Structure):
    _fields_ = [("packed_codes", ctypes.c_void_p), ("packed_code_bytes", ctypes.c_uint64),
                ("scales", ctypes.c_void_p), ("scale_count", ctypes.c_uint64)]


ERRORS = {1: "truncated", 2: "magic", 3: "version", 4: "stage", 5: "scale_count",
          6: "length", 7: "nonfinite", 8: "negative", 9: "geometry", 10: "prefix",
          11: "input", 12: "capacity"}


class OracleError(ValueError):
    def __init__(self, code: int):
        super().__init__(f"oracle rejected input: {ERRORS.get(code, code)}")
        self.code = code
        self.kind = ERRORS.get(code, str(code))


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} missing; run __graft_entry__.build()")
        L = ctypes.CDLL(str(LIB_PATH))
        u64, vp, i32 = ctypes.c_uint64, ctypes.c_void_p, ctypes.c_int
        L.hqo_crc32c.restype = ctypes.c_uint32
        L.hqo_crc32c.argtypes = [vp, ctypes.c_size_t, ctypes.c_uint32]
        L.hqo_half_to_float.restype = ctypes.c_float
        L.hqo_half_to_float.argtypes = [ctypes.c_uint16]
        L.hqo_decode_payload.restype = i32
        L.hqo_decode_payload.argtypes = [vp, ctypes.c_size_t, ctypes.c_uint16, u64,
                                         vp, u64, ctypes.POINTER(u64), vp, u64,
                                         ctypes.POINTER(u64)]
        for name in ("hqo_dequantize_stage", "hqo_dequantize_prefix"):
            getattr(L, name).restype = i32
            getattr(L, name).argtypes = [ctypes.POINTER(Geometry), ctypes.POINTER(Stage),
                                         ctypes.c_uint32, ctypes.c_uint32, vp]
        L.hqo_dequantize_mixed.restype = i32
        L.hqo_dequantize_mixed.argtypes = [ctypes.POINTER(Geometry), ctypes.POINTER(Stage),
                                           ctypes.c_uint32, vp, vp]
        L.hqo_linear_reference.restype = i32
        L.hqo_linear_reference.argtypes = [ctypes.POINTER(Geometry), ctypes.POINTER(Stage),
                                           ctypes.c_uint32, ctypes.c_uint32, vp, u64, vp, vp]
        L.hqo_linear_mixed.restype = i32
        L.hqo_linear_mixed.argtypes = [ctypes.POINTER(Geometry), ctypes.POINTER(Stage),
                                       ctypes.c_uint32, vp, vp, u64, vp, vp]
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


@dataclass
class Matrix:
    """Host progressive matrix: geometry + per-stage packed codes and FP32 scales."""
    geometry: tuple[int, int, int, int, int, int, int]
    codes: list[np.ndarray]
    scales: list[np.ndarray]   # float32, flat in [gr][gc][tile_rows][groups] order

    @property
    def rows(self) -> int:
        return self.geometry[0]

    @property
    def cols(self) -> int:
        return self.geometry[1]

    @property
    def stage_count(self) -> int:
        return len(self.codes)

    @property
    def grid(self) -> tuple[int, int]:
        g = self.geometry
        return g[2] // g[4], g[3] // g[5]

    def _c(self):
        geo = Geometry(*self.geometry)
        arr = (Stage * max(1, len(self.codes)))()
        keep = []
        for i, (c, s) in enumerate(zip(self.codes, self.scales)):
            c = np.ascontiguousarray(c, np.uint8)
            s = np.ascontiguousarray(s, np.float32).reshape(-1)
            keep += [c, s]
            arr[i] = Stage(c.ctypes.data, c.size, s.ctypes.data, s.size)
        return geo, arr, keep

    @staticmethod
    def from_quantized(q) -> "Matrix":
        return Matrix(tuple(q.geometry), [np.asarray(c, np.uint8) for c in q.codes],
                      [np.asarray(s, np.float16).astype(np.float32).reshape(-1) for s in q.scales])

    @staticmethod
    def from_payloads(geometry, payload_list: list[bytes]) -> "Matrix":
        g = geometry
        scale_count = (g[2] // g[4]) * (g[3] // g[5]) * g[4] * (g[5] // g[6])
        codes, scales = [], []
        for i, p in enumerate(payload_list):
            c, s = decode_payload(p, i, scale_count)
            codes.append(c)
            scales.append(s)
        return Matrix(tuple(geometry), codes, scales)


def crc32c(data: bytes, crc: int = 0) -> int:
    buf = ctypes.create_string_buffer(bytes(data), len(data))
    return lib().hqo_crc32c(buf, len(data), crc)


def half_to_float(bits: int) -> float:
    return lib().hqo_half_to_float(bits)


def decode_payload(payload: bytes, stage: int, scale_count: int) -> tuple[np.ndarray, np.ndarray]:
    buf = np.frombuffer(bytes(payload), np.uint8).copy()
    codes = np.zeros(max(1, len(payload)), np.uint8)
    scales = np.zeros(max(1, scale_count), np.float32)
    nc, ns = ctypes.c_uint64(), ctypes.c_uint64()
    rc = lib().hqo_decode_payload(_ptr(buf), len(payload), stage, scale_count, _ptr(codes),
                                  codes.size, ctypes.byref(nc), _ptr(scales), scales.size,
                                  ctypes.byref(ns))
    if rc:
        raise OracleError(rc)
    return codes[: nc.value].copy(), scales[: ns.value].copy()


def dequantize_prefix(m: Matrix, prefix: int) -> np.ndarray:
    geo, arr, _keep = m._c()
    out = np.zeros((m.rows, m.cols), np.float32)
    rc = lib().hqo_dequantize_prefix(ctypes.byref(geo), arr, m.stage_count, prefix, _ptr(out))
    if rc:
        raise OracleError(rc)
    return out


def dequantize_stage(m: Matrix, stage: int) -> np.ndarray:
    geo, arr, _keep = m._c()
    out = np.zeros((m.rows, m.cols), np.float32)
    rc = lib().hqo_dequantize_stage(ctypes.byref(geo), arr, m.stage_count, stage, _ptr(out))
    if rc:
        raise OracleError(rc)
    return out


def dequantize_mixed(m: Matrix, depth: np.ndarray) -> np.ndarray:
    geo, arr, _keep = m._c()
    d = np.ascontiguousarray(depth, np.uint8)
    out = np.zeros((m.rows, m.cols), np.float32)
    rc = lib().hqo_dequantize_mixed(ctypes.byref(geo), arr, m.stage_count, _ptr(d), _ptr(out))
    if rc:
        raise OracleError(rc)
    return out


def linear_reference(m: Matrix, x: np.ndarray, prefix: int, bias: np.ndarray | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, m.cols)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    geo, arr, _keep = m._c()
    out = np.zeros((x.shape[0], m.rows), np.float32)
    rc = lib().hqo_linear_reference(ctypes.byref(geo), arr, m.stage_count, prefix, _ptr(x),
                                    x.shape[0], _ptr(b), _ptr(out))
    if rc:
        raise OracleError(rc)
    return out


def linear_mixed(m: Matrix, x: np.ndarray, depth: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, m.cols)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    d = np.ascontiguousarray(depth, np.uint8)
    geo, arr, _keep = m._c()
    out = np.zeros((x.shape[0], m.rows), np.float32)
    rc = lib().hqo_linear_mixed(ctypes.byref(geo), arr, m.stage_count, _ptr(d), _ptr(x),
                                x.shape[0], _ptr(b), _ptr(out))
    if rc:
        raise OracleError(rc)
    return out


def stage_dense_np(m: Matrix, s: int) -> np.ndarray:
    """FP32 stage matrix (original shape), same exact products as the C oracle."""
    g = m.geometry
    rows, cols, rows_p, cols_p, tr, tc, grp = g
    raw = (m.codes[s][:, None] >> np.array([0, 2, 4, 6], np.uint8)[None, :]) & 3
    raw = raw.reshape(-1)[: rows_p * cols_p].astype(np.int8)
    codes = np.where(raw >= 2, raw - 4, raw).astype(np.float32).reshape(rows_p, cols_p)
    gr, gc = rows_p // tr, cols_p // tc
    sc = m.scales[s].reshape(gr, gc, tr, tc // grp)
    # expand to [rows_p, cols_p]: scale(row, col) = sc[row//tr, col//tc, row%tr, (col%tc)//grp]
    full = np.repeat(sc, grp, axis=3).reshape(gr, gc, tr, tc).transpose(0, 2, 1, 3).reshape(rows_p, cols_p)
    return (codes * full)[:rows, :cols]


def progressive_matmul_np(m: Matrix, x: np.ndarray, prefix: int, bias: np.ndarray | None = None) -> np.ndarray:
    """NumPy restatement of the reference's ``progressive_matmul``
    (src/harpq/quantization.py:352-406): each selected stage is decoded to dense FP32
    (``dequantize_stage``) and multiplied on its own (BLAS), the stage outputs accumulated in
    stage order into FP32 zeros, then the bias.  Test infrastructure and the NumPy CPU
    baseline; not a product path."""
    xs = np.asarray(x, np.float32).reshape(-1, m.cols)
    out = np.zeros((xs.shape[0], m.rows), np.float32)
    for s in range(prefix):
        out += xs @ stage_dense_np(m, s).T
    if bias is not None:
        out += np.asarray(bias, np.float32)
    return out


def dequantize_prefix_np(m: Matrix, prefix: int, depth: np.ndarray | None = None) -> np.ndarray:
    """Vectorised twin of hqo_dequantize_prefix / hqo_dequantize_mixed."""
    g = m.geometry
    out = np.zeros((g[0], g[1]), np.float32)
    stop = m.stage_count if depth is not None else prefix
    if depth is not None:
        gr, gc = m.grid
        d = np.asarray(depth, np.uint8).reshape(gr, gc)
        dfull = np.repeat(np.repeat(d, g[4], axis=0), g[5], axis=1)[: g[0], : g[1]]
    for s in range(stop):
        w = stage_dense_np(m, s)
        if depth is not None:
            w = np.where(dfull > s, w, np.float32(0.0))
        out += w
    return out


def have_reference() -> bool:
    return REF_LIB_PATH.exists()
