"""Failure detection on one GPU without a fault: a bounded device wait that runs out.

The fused all-gather's wait (hqb_gather_wait_ex) spins on per-rank flags that a peer raises
after its last output store.  Here no rank ever raises them: the wait must end after its
bound with HQB_DEVERR_TIMEOUT in the caller's flag word and the epoch advanced, the stream
must go on, and the context must stay usable (a GEMV right after is correct).  Nothing is
made to fault, trap or hang.
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from conftest import assert_close, plane_matrix, random_matrix  # noqa: E402


def test_gather_wait_runs_out_and_context_stays_usable():
    import harpq_b200 as hqb

    L = hqb.lib()
    world = 2
    flags = torch.zeros(hqb.MAX_PEERS, dtype=torch.int32, device="cuda")  # never raised
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    dev_flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    limit_ns = 50_000_000  # 50 ms
    t0 = time.perf_counter()
    assert L.hqb_gather_wait_ex(flags.data_ptr(), world, epoch.data_ptr(), dev_flags.data_ptr(), limit_ns,
                                stream) == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(dev_flags.item()) & hqb.DEVERR_TIMEOUT
    assert int(epoch.item()) == 1
    assert 0.04 <= waited < 2.0, waited
    # the context still runs work correctly
    rng = np.random.default_rng(8)
    m = random_matrix(rng, 256, 384)
    pm = plane_matrix(m)
    x = torch.from_numpy(rng.standard_normal((1, m.cols)).astype(np.float16)).cuda()
    y = pm.gemv(x, prefix=2, y_dtype=torch.float32).cpu().numpy()
    e = (x.double() @ pm.decode(2).double().T).cpu().numpy()
    assert_close(y, e, 2e-4, 2e-4, "GEMV after a wait that ran out")
    # flags raised for the next epoch: the wait ends at once, with no new error bit
    flags[:world] = 2
    dev_flags.zero_()
    assert L.hqb_gather_wait_ex(flags.data_ptr(), world, epoch.data_ptr(), dev_flags.data_ptr(), limit_ns,
                                stream) == 0
    torch.cuda.synchronize()
    assert int(dev_flags.item()) == 0
    assert int(epoch.item()) == 2


def test_gather_wait_rejects_bad_arguments():
    import harpq_b200 as hqb

    L = hqb.lib()
    buf = torch.zeros(16, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.hqb_gather_wait_ex(buf.data_ptr(), 0, buf.data_ptr(), None, 1000, st) == hqb.HQB_ERR_INVALID
    assert L.hqb_gather_wait_ex(buf.data_ptr(), 2, buf.data_ptr(), None, 0, st) == hqb.HQB_ERR_INVALID
    assert L.hqb_gather_wait_ex(None, 2, buf.data_ptr(), None, 1000, st) == hqb.HQB_ERR_INVALID
