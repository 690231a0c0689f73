"""Warp-level model of the depth-map range search of the stream-K kernel (CPU only).

With a per-tile depth map, each warp of a stream-K CTA finds its CTA's unit range
[floor(i*T/G), floor((i+1)*T/G)) in tiles itself (hqb_plane.cu, plan_row_of,
row_unit_tile, mixed_range): a 32-way search of the row plan with a ballot per round,
then an inclusive warp scan of one row's depths, 32 tiles per round.  This model runs
those steps lane by lane (ballot = the set of lanes whose predicate holds, shuffles =
reads of other lanes' values) and checks them against a direct scan of the map, on maps
with up to 600 tile rows (several search rounds) and 224 tile columns (several scan
rounds).  The kernels themselves are checked against the oracle by the -m gpu tests.
"""

from __future__ import annotations

import numpy as np
import pytest


def _plan(depth, stage_count):
    d = np.clip(depth.astype(np.int64), 1, stage_count)
    return np.concatenate([[0], np.cumsum(d.sum(axis=1))]), d


def _plan_row_of(plan, R, u):
    lo, hi = 0, R
    rounds = 0
    while hi - lo > 1:
        step = (hi - lo + 31) // 32
        le = [(lo + lane * step) < hi and plan[lo + lane * step] <= u for lane in range(32)]
        assert le[0]  # lane 0 always qualifies
        k = max(lane for lane in range(32) if le[lane])  # 31 - clz(ballot)
        lo += k * step
        hi = min(hi, lo + step)
        rounds += 1
    return lo, plan[lo], plan[lo + 1], rounds


def _row_unit_tile(d_row, off):
    C = len(d_row)
    before = 0
    for c0 in range(0, C, 32):
        d = [int(d_row[c0 + lane]) if c0 + lane < C else 0 for lane in range(32)]
        incl = list(d)
        o = 1
        while o < 32:  # shfl_up scan: each lane reads the value o lanes below, as it was
            prev = list(incl)
            for lane in range(o, 32):
                incl[lane] = prev[lane] + prev[lane - o]
            o <<= 1
        ballot = [before + incl[lane] > off for lane in range(32)]
        if any(ballot):
            k = ballot.index(True)  # ffs(ballot) - 1
            return c0 + k, off - before - (incl[k] - d[k])
        before += incl[31]
    raise AssertionError("unit beyond the row")


def _direct(dd, u):
    flat = dd.reshape(-1)
    cum = np.concatenate([[0], np.cumsum(flat)])
    t = int(np.searchsorted(cum, u, side="right") - 1)
    return t, int(u - cum[t])


@pytest.mark.parametrize("R,C,G,seed", [(86, 32, 296, 7), (600, 3, 296, 1), (8, 224, 296, 2), (33, 33, 64, 3),
                                        (1, 1, 296, 4), (512, 2, 148, 5)])
def test_ranges_match_a_direct_scan(R, C, G, seed):
    rng = np.random.default_rng(seed)
    depth = rng.integers(0, 6, size=(R, C)).astype(np.uint8)  # 0 and 5 exercise the clamp
    plan, dd = _plan(depth, 4)
    total = int(plan[R])
    ctas = min(total, G)
    covered = []
    max_rounds = 0
    for cta in range(ctas):
        u0, u1 = cta * total // ctas, (cta + 1) * total // ctas
        ends = []
        for u in (u0, u1 - 1):
            r, rb, re, rounds = _plan_row_of(plan, R, u)
            max_rounds = max(max_rounds, rounds)
            assert rb <= u < re
            c, s = _row_unit_tile(dd[r], u - rb)
            assert (r * C + c, s) == _direct(dd, u)
            assert 0 <= s < dd[r, c]
            ends.append((r * C + c, s))
        (t0, s0), (t_end, s_last) = ends
        # the CTA's units, tile by tile, with the stage masks the walk uses
        for t in range(t0, t_end + 1):
            d = int(dd.reshape(-1)[t])
            first = s0 if t == t0 else 0
            last = s_last if t == t_end else d - 1
            covered.extend((t, s) for s in range(first, last + 1))
    # every unit exactly once, in order
    assert covered == [(t, s) for t in range(R * C) for s in range(int(dd.reshape(-1)[t]))]
    if R > 32:
        assert max_rounds >= 2
