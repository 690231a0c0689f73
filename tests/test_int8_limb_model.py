"""Bit-level model of the int8-limb tensor-core form of the plane GEMV (CPU only).

The model runs one 16-row block of one 128x128 tile the way the kernels do:
* plane code words of lane (g, q): w0 = row g, columns 32q..32q+15; w1 = row g+8, same;
  w2 = row g, columns 32q+16..32q+31; w3 = row g+8, same; code + 2 at bits 2j;
* MMA m (0..3) takes the words ANDed with 0x03030303 << 2m as its u8 A registers
  (a0 = w0, a1 = w1, a2 = w2, a3 = w3), i.e. byte j holds (code+2)*4^m of column 4j+m;
* the s8 B registers come from a limb slot laid out as prep_i8_items writes it;
* the m16n8k32 fragment mapping is the PTX ISA's (A: rows g / g+8, k = 4q+i / 4q+16+i;
  B: k = 4q+i / 4q+16+i, n = g; C/D: row g / g+8, columns 2q, 2q+1);
* accumulators start from the bits of 1.5*2^23, the epilogue is fma(acc, L, K) then
  fma(sigma, v, y), and the lane quad is summed by two butterfly steps.
It checks the result against FP64 and that every stage of it is exact where the kernels
rely on exactness.  This pins the index and scaling arithmetic of the int8 form; the CUDA
kernels themselves are checked against the oracle by the -m gpu tests.
"""

from __future__ import annotations

import numpy as np
import pytest

LIMBS = 4
ACC_BIAS_BITS = 0x4B400000  # FP32 1.5 * 2^23


def _f32(v):
    return np.float32(v)


def _fma32(a, b, c):
    """FP32 fused multiply-add: exact product and sum (in FP64 here, exact for these
    operands), one rounding."""
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def _plane_words(codes):
    stored = (codes + 2).astype(np.uint64)
    words = np.zeros((32, 4), np.uint64)
    for lane in range(32):
        g, q = lane >> 2, lane & 3
        for i, (r, c0) in enumerate([(g, 32 * q), (g + 8, 32 * q), (g, 32 * q + 16), (g + 8, 32 * q + 16)]):
            words[lane, i] = sum(int(stored[r, c0 + j]) << (2 * j) for j in range(16))
    return words


def _limb_slot(x, batch):
    """prep_i8_items for one tile: x [batch][128] -> slot bytes and {L, K} per column."""
    slot = np.zeros(LIMBS * batch * 128, np.uint8)
    cst = np.zeros((8, 2), np.float32)
    for b in range(batch):
        v = x[b].astype(np.float32).reshape(32, 4)
        a = float(np.max(np.abs(v)))
        E = max(-90, min(100, int((np.float32(a).view(np.int32) >> 23) & 0xFF) - 126)) if a > 0 else 0
        assert a < 2.0 ** E
        sums = [0] * LIMBS
        for lane in range(32):
            base = (lane >> 3) * 32 + (lane & 7)
            for t in range(4):
                scaled = np.float64(v[lane, t]) * 2.0 ** (30 - E - 2 * t)  # exact power-of-2 scaling
                y = int(np.rint(scaled))  # round half to even, as __float2int_rn
                limbs = [0] * LIMBS
                for l in range(LIMBS - 1, 0, -1):
                    limbs[l] = ((y & 0xFF) ^ 0x80) - 0x80
                    y = (y - limbs[l]) >> 8
                limbs[0] = y
                assert -64 <= limbs[0] <= 64
                for l in range(LIMBS):
                    slot[(l * batch + b) * 128 + base + 8 * t] = limbs[l] & 0xFF
                    sums[l] += limbs[l] * 4 ** t
        for l in range(LIMBS):
            n = 2 * l + b
            L = _f32(2.0 ** (E - 6 - 8 * l))
            bias_plus = _f32(12582912.0 + 2 * sums[l])
            assert float(bias_plus) == 12582912.0 + 2 * sums[l]  # exact in FP32
            cst[n] = (L, -bias_plus * L)
    return slot, cst


def _bytes(w):
    return [(int(w) >> (8 * i)) & 0xFF for i in range(4)]


def _mma_m16n8k32(a_regs, b_regs, c):
    A = np.zeros((16, 32), np.int64)
    B = np.zeros((32, 8), np.int64)
    for lane in range(32):
        g, q = lane >> 2, lane & 3
        for i, (r, k0) in enumerate([(g, 4 * q), (g + 8, 4 * q), (g, 4 * q + 16), (g + 8, 4 * q + 16)]):
            A[r, k0:k0 + 4] = _bytes(a_regs[lane][i])
        for i, k0 in enumerate([4 * q, 4 * q + 16]):
            B[k0:k0 + 4, g] = [v - 256 if v >= 128 else v for v in _bytes(b_regs[lane][i])]
    D = A @ B
    assert np.abs(D).max() < 2 ** 31
    out = []
    for lane in range(32):
        g, q = lane >> 2, lane & 3
        out.append([c[lane][0] + D[g, 2 * q], c[lane][1] + D[g, 2 * q + 1],
                    c[lane][2] + D[g + 8, 2 * q], c[lane][3] + D[g + 8, 2 * q + 1]])
    return out


def _row_block(codes, sigma, x):
    batch = x.shape[0]
    words = _plane_words(codes)
    slot, cst = _limb_slot(x, batch)
    slot_words = slot.view(np.uint32)
    acc = [[ACC_BIAS_BITS] * 4 for _ in range(32)]
    for m in range(4):
        mask = 0x03030303 << (2 * m)
        a = [[int(words[lane, i]) & mask for i in range(4)] for lane in range(32)]
        b = []
        for lane in range(32):
            g, q = lane >> 2, lane & 3
            entry = (0 if g & 1 else g >> 1) if batch == 1 else g
            off = (entry * 128 + q * 32) // 4
            b.append([int(slot_words[off + 2 * m]), int(slot_words[off + 2 * m + 1])])
        acc = _mma_m16n8k32(a, b, acc)
    y = np.zeros((32, 4), np.float32)
    for lane in range(32):
        g, q = lane >> 2, lane & 3
        for e in range(4):
            j = e & 1
            if batch == 1 and j:
                continue
            bits = acc[lane][e]
            assert abs(bits - ACC_BIAS_BITS) < 2 ** 22  # FP32 reading of the biased sum is exact
            accf = np.array([bits], np.uint32).view(np.float32)[0]
            L, K = cst[2 * q + j]
            v = _fma32(accf, L, K)
            exact = (float(accf) - 12582912.0) * float(L) + float(K) + 12582912.0 * float(L)
            assert float(v) == exact  # the first FMA is exact
            s = sigma[g] if e < 2 else sigma[g + 8]
            y[lane, e] = _fma32(s, v, y[lane, e])
    for e in range(4):
        col = y[:, e].copy()
        col = np.array([np.float32(col[l] + col[l ^ 1]) for l in range(32)])
        col = np.array([np.float32(col[l] + col[l ^ 2]) for l in range(32)])
        y[:, e] = col
    return y


@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("case", ["plain", "outliers", "extremes", "fp32_wide"])
def test_int8_limb_row_block_model(batch, case):
    rng = np.random.default_rng({"plain": 1, "outliers": 2, "extremes": 3, "fp32_wide": 4}[case] + 10 * batch)
    codes = rng.integers(-2, 2, size=(16, 128))
    sigma = rng.uniform(0.002, 0.05, size=16).astype(np.float16).astype(np.float32)
    x = rng.standard_normal((batch, 128)).astype(np.float16).astype(np.float32)
    if case == "outliers":
        x[:, ::17] *= 20
    elif case == "extremes":
        x[0, :64] = (rng.standard_normal(64) * 2.0 ** -20).astype(np.float16)  # FP16 subnormals
        x[0, 70] = 65504.0
    elif case == "fp32_wide":  # FP32 activations spanning 1e-6..1e6 in the tile
        x = (np.sign(rng.standard_normal((batch, 128))) * 10.0 ** rng.uniform(-6, 6, size=(batch, 128)))
        x = x.astype(np.float32)
    y = _row_block(codes, sigma, x)
    w = (codes * sigma[:, None]).astype(np.float64)
    ref = w @ x.T.astype(np.float64)  # [16][batch]
    # each x is rounded to at most 2^-25 of its tile's largest |x|; the FP32 epilogue adds
    # rounding relative to the sum of |w*x|
    quant = np.abs(w).sum(axis=1)[:, None] * (2.0 ** -25 * np.abs(x).max(axis=1))[None, :]
    fp32 = 1e-6 * (np.abs(w) @ np.abs(x.T).astype(np.float64))
    for lane in range(0, 32, 4):  # quad position 0 holds the summed rows
        g = lane >> 2
        for b in range(batch):
            for row, e in ((g, b), (g + 8, 2 + b)):
                err = abs(float(y[lane, e]) - ref[row, b])
                assert err <= quant[row, b] + fp32[row, b] + 1e-12, (case, batch, row, b, err)
