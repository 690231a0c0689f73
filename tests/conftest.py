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
