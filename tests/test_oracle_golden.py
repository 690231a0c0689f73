"""CPU: pin the C oracle and the NumPy encoder restatement to the reference.

Known-answer vectors come from the reference's own tests:
* CRC32C("123456789") == 0xE3069283 and incremental update (stage_codec_test.cpp:76-91)
* byte 0x4E -> codes [-2,-1,0,1]; [-2,-1,0,1,1] packs to 0x4E,0x01
  (stage_codec_test.cpp:148-161, test_quantization.py:19-25)
* raw FP16 0x0001 -> 2^-24, 0x7BFF -> 65504 (progressive_gemv_test.cu:473-476)
* the 5x9 golden fixture: exact prefix weights, outputs within 1e-6
  (stage_codec_test.cpp:163-179)
* payload validation failures (stage_codec_test.cpp:93-146)
"""

from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest

from conftest import SEEDED_NAMES, load_seeded
from oracle import oracle as orc
from oracle import quantize as qz


def test_crc32c_known_answers(native_golden):
    assert orc.crc32c(b"123456789") == 0xE3069283
    assert orc.crc32c(b"56789", orc.crc32c(b"1234")) == 0xE3069283
    assert orc.crc32c(b"") == 0
    for i, p in enumerate(native_golden["payloads"]):
        assert orc.crc32c(p.tobytes()) == int(native_golden["crc32c"][i])


def test_half_to_float_known_answers():
    assert orc.half_to_float(0x0001) == 2.0 ** -24
    assert orc.half_to_float(0x7BFF) == 65504.0
    assert orc.half_to_float(0x3C00) == 1.0
    assert orc.half_to_float(0xC000) == -2.0
    for bits in range(0, 0x7C00, 7):  # every finite positive class, sampled
        assert np.float32(orc.half_to_float(bits)) == np.array([bits], np.uint16).view(np.float16).astype(np.float32)[0]


def test_int2_layout_known_answers():
    assert list(qz.pack_codes(np.array([-2, -1, 0, 1, 1], np.int8))) == [0x4E, 0x01]
    m = orc.Matrix((1, 4, 1, 4, 1, 4, 4), [np.array([0x4E], np.uint8)], [np.array([1.0], np.float32)])
    np.testing.assert_array_equal(orc.dequantize_prefix(m, 1), [[-2.0, -1.0, 0.0, 1.0]])


def test_golden_prefix_weights_exact_and_outputs(native_golden, golden_matrix):
    z = native_golden
    for p in range(5):
        w = orc.dequantize_prefix(golden_matrix, p)
        assert w.tobytes() == z["prefix_weights"][p].tobytes(), f"prefix {p} weights"
        y = orc.linear_reference(golden_matrix, z["inputs"], p, z["bias"])
        np.testing.assert_allclose(y, z["prefix_outputs"][p], rtol=0, atol=1e-6)
        # the fixture fixes scalar order: the oracle reproduces it exactly
        assert y.tobytes() == z["prefix_outputs"][p].tobytes()


def test_numpy_twin_matches_c_oracle(golden_matrix):
    for p in range(5):
        assert orc.dequantize_prefix_np(golden_matrix, p).tobytes() == orc.dequantize_prefix(golden_matrix, p).tobytes()


def test_payload_validation(native_golden):
    good = native_golden["payloads"][0].tobytes()
    count = 32
    orc.decode_payload(good, 0, count)

    def reject(buf, kind, stage=0, n=count):
        with pytest.raises(orc.OracleError) as e:
            orc.decode_payload(buf, stage, n)
        assert e.value.kind == kind

    reject(good[:19], "truncated")
    reject(b"\x00" + good[1:], "magic")
    reject(good[:8] + b"\x02" + good[9:], "version")
    reject(good, "stage", stage=1)
    reject(good[:-1], "length")
    reject(good + b"\x00", "length")
    reject(good[:16] + b"\x07" + good[17:], "scale_count")
    first = 20 + 32
    neg = bytearray(good)
    neg[first + 1] |= 0x80
    if struct.unpack_from("<H", good, first)[0] & 0x7FFF:
        reject(bytes(neg), "negative")
    nan = bytearray(good)
    nan[first:first + 2] = b"\x00\x7e"
    reject(bytes(nan), "nonfinite")


def test_oracle_rejects_bad_geometry_and_prefix(golden_matrix):
    with pytest.raises(orc.OracleError):
        orc.dequantize_prefix(golden_matrix, 5)
    bad = orc.Matrix(golden_matrix.geometry[:3] + (15,) + golden_matrix.geometry[4:],
                     golden_matrix.codes, golden_matrix.scales)
    with pytest.raises(orc.OracleError):
        orc.dequantize_prefix(bad, 1)
    x = np.zeros((1, golden_matrix.cols), np.float32)
    x[0, 0] = np.inf
    with pytest.raises(orc.OracleError):
        orc.linear_reference(golden_matrix, x, 1)


@pytest.mark.parametrize("name", SEEDED_NAMES)
def test_seeded_fixture_decode_matches_reference_digest(name):
    m, payloads, z = load_seeded(name)
    for i, p in enumerate(payloads):
        assert orc.crc32c(p) == int(z["crc32c"][i])
    for p in range(5):
        w = orc.dequantize_prefix(m, p)
        assert hashlib.sha256(w.tobytes()).digest() == z["prefix_sha256"][p].tobytes(), f"prefix {p}"
    if "prefix4_weights" in z.files:
        assert orc.dequantize_prefix(m, 4).tobytes() == z["prefix4_weights"].tobytes()


@pytest.mark.parametrize("name", SEEDED_NAMES)
def test_seeded_fixture_linear_matches_reference_numpy(name):
    m, _, z = load_seeded(name)
    for p in range(5):
        y = orc.linear_reference(m, z["x"], p, z["bias"])
        # the reference's NumPy progressive_matmul dispatches to BLAS: compare
        # within its documented tolerance (generate_native_golden.py:96-101)
        np.testing.assert_allclose(y, z["prefix_outputs"][p], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", SEEDED_NAMES)
def test_numpy_matmul_restatement_matches_reference_outputs(name):
    """progressive_matmul_np (the NumPy CPU baseline) against the reference's own
    progressive_matmul outputs stored in the fixture (same decode, BLAS matmul per stage)."""
    m, _, z = load_seeded(name)
    for p in range(5):
        y = orc.progressive_matmul_np(m, z["x"], p, z["bias"])
        np.testing.assert_allclose(y, z["prefix_outputs"][p], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", SEEDED_NAMES)
def test_numpy_encoder_restatement_is_byte_identical(name):
    _, payloads, z = load_seeded(name)
    q = qz.quantize(z["weights"])
    assert qz.payloads(q) == payloads


def test_mixed_depth_oracle_consistency():
    _, _, z = load_seeded("grid2")
    m, _, _ = load_seeded("grid2")
    gr, gc = m.grid
    rng = np.random.default_rng(5)
    depth = rng.integers(1, 5, size=(gr, gc), dtype=np.uint8)
    w = orc.dequantize_mixed(m, depth)
    assert w.tobytes() == orc.dequantize_prefix_np(m, 0, depth=depth).tobytes()
    # uniform depth map == uniform prefix, bit for bit
    for p in range(1, 5):
        u = np.full((gr, gc), p, np.uint8)
        assert orc.dequantize_mixed(m, u).tobytes() == orc.dequantize_prefix(m, p).tobytes()
        y1 = orc.linear_mixed(m, z["x"], u, z["bias"])
        y2 = orc.linear_reference(m, z["x"], p, z["bias"])
        assert y1.tobytes() == y2.tobytes()
