"""Shared pytest setup: the ``gpu`` marker, import paths and golden fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
for p in (REPO, REPO / "harp-q_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_seeded(name: str):
    """Seeded reference fixture -> (oracle Matrix, payload list, npz)."""
    from oracle import oracle as orc

    z = np.load(GOLDEN / f"seeded_{name}.npz")
    raw = z["payloads"].tobytes()
    payloads, off = [], 0
    for n in z["payload_lengths"]:
        payloads.append(raw[off: off + int(n)])
        off += int(n)
    geom = tuple(int(v) for v in z["geometry"])
    return orc.Matrix.from_payloads(geom, payloads), payloads, z


SEEDED_NAMES = ("tile1", "ragged", "grid2")


@pytest.fixture(scope="session")
def native_golden():
    return np.load(GOLDEN / "native_golden.npz")


@pytest.fixture(scope="session")
def golden_matrix(native_golden):
    from oracle import oracle as orc

    z = native_golden
    geom = tuple(int(v) for v in z["geometry"])
    ss = [int(v) for v in z["scale_shape"]]
    count = ss[0] * ss[1] * ss[2] * ss[3]
    codes, scales = [], []
    for i, p in enumerate(z["payloads"]):
        c, s = orc.decode_payload(p.tobytes(), i, count)
        codes.append(c)
        scales.append(s)
    return orc.Matrix(geom, codes, scales)


def device_stages(m, device="cuda"):
    """oracle.Matrix -> (codes uint8, FP16 scale bits int16, FP32 scales) CUDA tensors per stage."""
    import torch

    codes, bits, f32 = [], [], []
    for c, s in zip(m.codes, m.scales):
        codes.append(torch.from_numpy(np.ascontiguousarray(c, np.uint8)).to(device))
        s32 = np.ascontiguousarray(s, np.float32)
        bits.append(torch.from_numpy(s32.astype(np.float16).view(np.int16)).to(device))
        f32.append(torch.from_numpy(s32).to(device))
    return codes, bits, f32


def plane_matrix(m, device="cuda"):
    import harpq_b200 as hqb

    codes, bits, _ = device_stages(m, device)
    return hqb.PlaneMatrix.from_stages(m.rows, m.cols, codes, bits)


def random_matrix(rng, rows, cols, tile=(128, 128), group=128, stages=4, scale_exp=(-9, -4)):
    """Random int2 codes and FP16-exact scales (not from the quantizer)."""
    from oracle import oracle as orc

    rows_p = -(-rows // tile[0]) * tile[0]
    cols_p = -(-cols // tile[1]) * tile[1]
    nbytes = -(-rows_p * cols_p // 4)
    nscale = (rows_p // tile[0]) * (cols_p // tile[1]) * tile[0] * (tile[1] // group)
    codes = [rng.integers(0, 256, nbytes, dtype=np.uint8) for _ in range(stages)]
    scales = []
    for _ in range(stages):
        mant = rng.integers(0, 1024, nscale)
        ex = rng.integers(scale_exp[0], scale_exp[1] + 1, nscale)
        scales.append(np.ldexp(1.0 + mant / 1024.0, ex).astype(np.float16).astype(np.float32))
    return orc.Matrix((rows, cols, rows_p, cols_p, tile[0], tile[1], group), codes, scales)


def assert_close(actual, expected, atol, rtol, what=""):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    assert actual.shape == expected.shape, what
    assert np.all(np.isfinite(actual)), f"{what}: non-finite output"
    err = np.abs(actual - expected)
    tol = atol + rtol * np.abs(expected)
    bad = np.argwhere(err > tol)
    assert bad.size == 0, (f"{what}: {len(bad)} elements out of tolerance; first {tuple(bad[0])}: "
                           f"got {actual[tuple(bad[0])]}, want {expected[tuple(bad[0])]}")


def rel_l2(actual, expected) -> float:
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))
