"""CPU, world size 2 (gloo): the output-row sharding plan and all-gather assembly used by
the multi-GPU path.  Each rank evaluates its tile-row shard with the oracle, the ranks
all-gather padded slices, and the reassembled output must equal the unsharded oracle
output bit for bit (row sharding does not change any row's arithmetic)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, rows, cols, q):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "harp-q_b200"), str(root / "tests")]
    import harpq_b200 as hqb
    from conftest import random_matrix
    from oracle import oracle as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = random_matrix(np.random.default_rng(rows + cols), rows, cols)
        x = np.random.default_rng(1).standard_normal((1, cols)).astype(np.float32)
        r0, n = hqb.shard_rows(rows, world, rank)
        codes, bits = hqb.slice_stage_rows(m.codes, [s.astype(np.float16) for s in m.scales], cols, r0, n)
        sub = orc.Matrix((n, cols, -(-n // 128) * 128, m.geometry[3], 128, 128, 128), list(codes),
                         [b.astype(np.float32) for b in bits])
        pad = hqb.shard_pad_rows(rows, world)
        local = np.zeros(pad, np.float32)
        local[:n] = orc.linear_reference(sub, x, 4)[0]
        gathered = torch.empty(world * pad)
        dist.all_gather_into_tensor(gathered, torch.from_numpy(local))
        if rank == 0:
            parts = []
            for r in range(world):
                rr0, rn = hqb.shard_rows(rows, world, r)
                assert rr0 == sum(len(p) for p in parts)
                parts.append(gathered[r * pad: r * pad + rn].numpy())
            full = np.concatenate(parts)
            want = orc.linear_reference(m, x, 4)[0]
            q.put(full.tobytes() == want.tobytes())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows,world", [(1000, 2), (384, 2), (130, 2)])
def test_row_sharded_gather_matches_unsharded(rows, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, 200, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) is True


def test_shard_plan_covers_rows_once():
    import harpq_b200 as hqb

    for rows in (1, 127, 128, 129, 4096, 11008, 28672):
        for world in (1, 2, 4, 8):
            spans = [hqb.shard_rows(rows, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (a0, an), (b0, _) in zip(spans, spans[1:]):
                assert a0 + an == b0 and a0 % 128 == 0
            assert sum(n for _, n in spans) == rows
            assert max(n for _, n in spans) <= hqb.shard_pad_rows(rows, world)
