"""CPU: the C restatement against the reference's own C++ decoder (oracle/_ref).

oracle/_ref/libharpq_ref.so is native/src/stage_codec.cpp from the reference,
compiled in place by oracle/build.py.  These tests run wherever that binary
exists (this container after build(); it also travels to the GPU box).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import SEEDED_NAMES, load_seeded
from oracle import oracle as orc
from oracle import refcpu

pytestmark = pytest.mark.skipif(not refcpu.available(), reason="oracle/_ref not built")


def _random_matrix(rng, rows, cols, tile=(128, 128), group=128, stages=4):
    rows_p = -(-rows // tile[0]) * tile[0]
    cols_p = -(-cols // tile[1]) * tile[1]
    nbytes = -(-rows_p * cols_p // 4)
    nscale = (rows_p // tile[0]) * (cols_p // tile[1]) * tile[0] * (tile[1] // group)
    codes = [rng.integers(0, 256, nbytes, dtype=np.uint8) for _ in range(stages)]
    scales = [rng.integers(0, 0x7C00, nscale).astype(np.uint16).view(np.float16).astype(np.float32)
              * np.float32(1.0) for _ in range(stages)]
    return orc.Matrix((rows, cols, rows_p, cols_p, tile[0], tile[1], group), codes, scales)


@pytest.mark.parametrize("shape,tile,group", [((37, 70), (16, 32), 8), ((130, 259), (128, 128), 128),
                                              ((5, 9), (4, 8), 4), ((3, 513), (4, 128), 128)])
def test_decode_and_linear_bit_identical(shape, tile, group):
    rng = np.random.default_rng(sum(shape))
    m = _random_matrix(rng, *shape, tile=tile, group=group)
    ref = refcpu.RefMatrix(m)
    x = rng.standard_normal((2, shape[1])).astype(np.float32)
    bias = rng.standard_normal(shape[0]).astype(np.float32)
    for p in range(5):
        assert orc.dequantize_prefix(m, p).tobytes() == ref.dequantize_prefix(p).tobytes()
        assert orc.linear_reference(m, x, p, bias).tobytes() == ref.linear(x, p, bias).tobytes()


@pytest.mark.parametrize("name", SEEDED_NAMES)
def test_seeded_fixtures_against_reference(name):
    m, payloads, z = load_seeded(name)
    ref = refcpu.RefMatrix(m)
    for p in range(5):
        assert orc.dequantize_prefix(m, p).tobytes() == ref.dequantize_prefix(p).tobytes()
        assert orc.linear_reference(m, z["x"], p, z["bias"]).tobytes() == \
            ref.linear(z["x"], p, z["bias"]).tobytes()


def test_payload_decoder_matches_reference(native_golden):
    import ctypes

    ss = np.array(native_golden["scale_shape"], np.uint64)
    for i, p in enumerate(native_golden["payloads"]):
        codes = np.zeros(32, np.uint8)
        scales = np.zeros(32, np.float32)
        rc = refcpu.lib().hqr_decode_payload(p.ctypes.data, p.size, i, ss.ctypes.data,
                                             codes.ctypes.data, scales.ctypes.data)
        assert rc == 0
        c2, s2 = orc.decode_payload(p.tobytes(), i, 32)
        assert codes.tobytes() == c2.tobytes() and scales.tobytes() == s2.tobytes()
        assert refcpu.lib().hqr_crc32c(p.ctypes.data, p.size, 0) == orc.crc32c(p.tobytes())
    del ctypes


def test_row_shards_reassemble_reference():
    rng = np.random.default_rng(3)
    m = _random_matrix(rng, 300, 256)
    x = rng.standard_normal((1, 256)).astype(np.float32)
    whole = refcpu.RefMatrix(m).linear(x, 3)
    sharded = refcpu.ShardedReference(m, 3)
    try:
        assert sharded.linear(x, 3).tobytes() == whole.tobytes()
    finally:
        sharded.close()
