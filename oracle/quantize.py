"""TEST INFRASTRUCTURE ONLY — NumPy restatement of the reference's progressive encoder.

It produces the stage payloads every parity test and the CPU baseline feed to the
path under test, on machines where the reference package itself is absent.  Its
output is pinned byte-for-byte to the reference encoder by tests/golden (the
fixtures there were made by running the reference's own ``quantize_progressive``
and ``encode_stage_payload``).

Restated from the reference (src/harpq/quantization.py, src/harpq/matrix_codec.py):

* ``pack_codes``      — quantization.py:32-60   (4 codes per byte, LSB first)
* ``to_groups`` / ``from_groups`` — quantization.py:434-463
* ``fit_groups``      — quantization.py:466-521 (LS scale fit, 4 iterations,
                        FP16 scale, codes re-picked against the stored scale)
* ``quantize``        — quantization.py:228-309 (residual stages)
* ``stage_payload``   — matrix_codec.py:17-18, :57-73 (HQSTAGE wire format)

The arithmetic (dtypes, the FP64 reductions, rounding, clipping) follows the
reference step for step, because the produced codes must be identical.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass
from math import ceil

import numpy as np

STAGE_HEADER = struct.Struct("<8sHHII")
STAGE_MAGIC = b"HQSTAGE\x00"


def pack_codes(codes: np.ndarray) -> np.ndarray:
    """Signed int2 values in [-2, 1] -> bytes, value i at bits 2*(i%4)."""
    flat = np.asarray(codes).reshape(-1)
    if flat.size and (flat.min() < -2 or flat.max() > 1):
        raise ValueError("int2 codes must lie in [-2, 1]")
    two_bit = (flat.astype(np.int8) & 0x03).astype(np.uint8)
    pad = (-two_bit.size) % 4
    if pad:
        two_bit = np.concatenate([two_bit, np.zeros(pad, np.uint8)])
    quads = two_bit.reshape(-1, 4)
    out = quads[:, 0] | (quads[:, 1] << 2) | (quads[:, 2] << 4) | (quads[:, 3] << 6)
    return np.ascontiguousarray(out.astype(np.uint8))


def unpack_codes(packed: np.ndarray, count: int) -> np.ndarray:
    raw = (packed[:, None] >> np.array([0, 2, 4, 6], np.uint8)[None, :]) & 3
    raw = raw.reshape(-1)[:count].astype(np.int8)
    return np.where(raw >= 2, raw - 4, raw).astype(np.int8)


def to_groups(m: np.ndarray, tile: tuple[int, int], group: int) -> np.ndarray:
    tr, tc = tile
    gr, gc = m.shape[0] // tr, m.shape[1] // tc
    return m.reshape(gr, tr, gc, tc).transpose(0, 2, 1, 3).reshape(gr, gc, tr, tc // group, group)


def from_groups(blocks: np.ndarray, padded: tuple[int, int], tile: tuple[int, int]) -> np.ndarray:
    tr, tc = tile
    gr, gc = padded[0] // tr, padded[1] // tc
    return np.ascontiguousarray(blocks.reshape(gr, gc, tr, tc).transpose(0, 2, 1, 3).reshape(padded))


def fit_groups(blocks: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Least-squares int2 fit of every group; returns (codes int8, FP16 scales)."""
    shape = blocks.shape
    w = np.ascontiguousarray(blocks.reshape(-1, shape[-1]), dtype=np.float32)
    peak = np.max(np.abs(w), axis=1)
    s = np.where(peak > 0, peak / np.float32(1.5), 0).astype(np.float32)
    w64 = w.astype(np.float64)
    for _ in range(4):
        q = np.zeros_like(w)
        np.divide(w, s[:, None], out=q, where=s[:, None] != 0)
        c = np.clip(np.rint(q), -2, 1).astype(np.int8)
        c64 = c.astype(np.float64)
        num = np.sum(w64 * c64, axis=1)
        den = np.sum(c64 ** 2, axis=1)
        fit = np.divide(num, den, out=np.zeros_like(num), where=den != 0)
        s = np.where(den != 0, fit, s).astype(np.float32)
        s = np.maximum(s, np.float32(0.0))
    if np.any(s > np.finfo(np.float16).max):
        raise OverflowError("group scale exceeds FP16")
    s16 = s.astype(np.float16)
    if not np.all(np.isfinite(s16)):
        raise OverflowError("group scale exceeds FP16")
    exact = s16.astype(np.float32)
    q = np.zeros_like(w)
    np.divide(w, exact[:, None], out=q, where=exact[:, None] != 0)
    c = np.clip(np.rint(q), -2, 1).astype(np.int8)
    return (np.ascontiguousarray(c.reshape(shape), dtype=np.int8),
            np.ascontiguousarray(s16.reshape(shape[:-1]), dtype=np.float16))


@dataclass
class Quantized:
    original_shape: tuple[int, int]
    padded_shape: tuple[int, int]
    tile_shape: tuple[int, int]
    group_size: int
    codes: list[np.ndarray]      # packed uint8 per stage
    scales: list[np.ndarray]     # float16 [gr, gc, tile_rows, groups] per stage

    @property
    def geometry(self) -> tuple[int, int, int, int, int, int, int]:
        return (self.original_shape[0], self.original_shape[1], self.padded_shape[0],
                self.padded_shape[1], self.tile_shape[0], self.tile_shape[1], self.group_size)


def quantize(weights: np.ndarray, tile: tuple[int, int] = (128, 128), group: int = 128,
             stages: int = 4) -> Quantized:
    m = np.ascontiguousarray(np.asarray(weights), dtype=np.float32)
    if m.ndim != 2 or 0 in m.shape or not np.all(np.isfinite(m)):
        raise ValueError("weights must be a finite non-empty 2-D matrix")
    if tile[1] % group != 0 or not 1 <= stages <= 4:
        raise ValueError("invalid tile/group/stage geometry")
    padded = tuple(ceil(n / t) * t for n, t in zip(m.shape, tile))
    residual = np.zeros(padded, np.float32)
    residual[: m.shape[0], : m.shape[1]] = m
    codes_out, scales_out = [], []
    for _ in range(stages):
        c, s = fit_groups(to_groups(residual, tile, group))
        recon = c.astype(np.float32) * s[..., None].astype(np.float32)
        residual -= from_groups(recon, padded, tile)
        codes_out.append(pack_codes(from_groups(c, padded, tile)))
        scales_out.append(s)
    return Quantized((int(m.shape[0]), int(m.shape[1])), (int(padded[0]), int(padded[1])),
                     (int(tile[0]), int(tile[1])), int(group), codes_out, scales_out)


def stage_payload(codes: np.ndarray, scales: np.ndarray, stage_index: int) -> bytes:
    body = np.ascontiguousarray(codes, np.uint8).tobytes()
    tail = np.ascontiguousarray(scales, dtype="<f2").tobytes()
    return STAGE_HEADER.pack(STAGE_MAGIC, 1, stage_index, len(body), scales.size) + body + tail


def payloads(q: Quantized) -> list[bytes]:
    return [stage_payload(c, s, i) for i, (c, s) in enumerate(zip(q.codes, q.scales))]
