"""Fused all-gather of row-sharded GEMV outputs over peer memory (two GPUs of one node).

Each rank holds a 128-row-aligned row shard of the same layer, runs hqb_gemv_gather so
its outputs land in every rank's gathered buffer, waits with hqb_gather_wait, and checks
the gathered vector against the unsharded GEMV computed locally (FP32 contract), over
several steps (the flag epochs advance).  Needs at least two GPUs; skipped otherwise.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q) -> None:
    try:
        import sys
        from pathlib import Path

        repo = Path(__file__).resolve().parents[1]
        sys.path[:0] = [str(repo), str(repo / "harp-q_b200"), str(repo / "tests")]
        import torch.distributed as dist
        import harpq_b200 as hqb
        from conftest import plane_matrix, random_matrix

        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(31)
        m = random_matrix(rng, 700, 1000)  # same matrix on every rank
        full = plane_matrix(m)
        r0, nrows = hqb.shard_rows(m.rows, world, rank)
        slot = hqb.shard_pad_rows(m.rows, world)
        from conftest import device_stages

        codes, bits, _ = device_stages(m)
        codes, bits = hqb.slice_stage_rows(codes, bits, m.cols, r0, nrows)
        shard = hqb.PlaneMatrix.from_stages(nrows, m.cols, [c.contiguous() for c in codes],
                                            [b.contiguous() for b in bits])
        g = hqb.Gather(slot, batch=2, y_dtype=torch.float32)
        gen = torch.Generator(device="cuda").manual_seed(5)
        errors = []
        for step in range(3):
            x = torch.randn(2, m.cols, device="cuda", generator=gen).half()
            shard.gemv_gather(x, g, prefix=1 + step)
            g.wait()
            want = full.gemv(x, prefix=1 + step, y_dtype=torch.float32)
            got = g.out.view(2, world, slot)
            for r in range(world):
                rr0, rn = hqb.shard_rows(m.rows, world, r)
                diff = (got[:, r, :rn] - want[:, rr0:rr0 + rn]).abs()
                tol = 2e-4 + 2e-4 * want[:, rr0:rr0 + rn].abs()
                if not bool((diff <= tol).all()):
                    errors.append(f"step {step} slice {r}: max diff {float(diff.max())}")
        torch.cuda.synchronize()
        errors += [f"device flags {int(g.device_flags.item())}"] if int(g.device_flags.item()) else []
        dist.barrier()
        g.close()
        dist.destroy_process_group()
        q.put((rank, errors))
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, [repr(exc)]))


def test_fused_gather_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, errors = q.get(timeout=240)
            results[rank] = errors
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert results == {0: [], 1: []}, results
