"""GPU: a decode step as one library call -- hqb_gemv_batch (eager) and hqb_step_* (the calls
captured once into a CUDA graph) -- gives the bytes of the same GEMVs called one by one, and
a captured step keeps working as its inputs are refilled in place."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from conftest import plane_matrix, random_matrix  # noqa: E402


def test_step_batch_and_graph_match_single_calls():
    import harpq_b200 as hqb

    rng = np.random.default_rng(2024)
    shapes = [(768, 512), (300, 512), (1024, 1000), (200, 11008)]
    pms = [plane_matrix(random_matrix(rng, r, c)) for r, c in shapes]
    xs = [torch.from_numpy(rng.standard_normal((1, c)).astype(np.float16)).cuda() for _, c in shapes]
    ys = [torch.empty(1, r, dtype=torch.float16, device="cuda") for r, _ in shapes]
    ws = hqb.Workspace(max(pm.workspace_bytes(1, hqb.F16) for pm in pms))
    prefixes = [1, 2, 3, 4]
    ref = [pm.gemv(x, prefix=p, y_dtype=torch.float16, workspace=ws) for pm, x, p in zip(pms, xs, prefixes)]
    calls = [(pm, x, p, y, hqb.FLAG_PDL) for pm, x, p, y in zip(pms, xs, prefixes, ys)]
    for graph in (False, True):
        step = hqb.Step(calls, ws, graph=graph)
        for y in ys:
            y.fill_(float("nan"))
        step.run()
        torch.cuda.synchronize()
        for a, b in zip(ys, ref):
            assert torch.equal(a, b), f"graph={graph}"
        # inputs refilled in place: the captured step reads the new values
        for x in xs:
            x.mul_(-1)
        step.run()
        torch.cuda.synchronize()
        for a, pm, x, p in zip(ys, pms, xs, prefixes):
            assert torch.equal(a, pm.gemv(x, prefix=p, y_dtype=torch.float16, workspace=ws))
        for x in xs:
            x.mul_(-1)
        step.close()
    assert ws.error_flags() == 0


def test_step_rejects_an_invalid_call_and_enqueues_nothing_after_it():
    import harpq_b200 as hqb

    rng = np.random.default_rng(3)
    pm = plane_matrix(random_matrix(rng, 256, 256, stages=2))
    x = torch.randn(1, 256, device="cuda").half()
    y = torch.empty(1, 256, dtype=torch.float16, device="cuda")
    ws = pm.workspace(1)
    with pytest.raises(hqb.HQBError) as e:
        hqb.Step([(pm, x, 3, y, 0)], ws)  # prefix 3 > stage count 2
    assert e.value.status == hqb.HQB_ERR_INVALID
    with pytest.raises(hqb.HQBError):
        hqb.Step([(pm, x, 3, y, 0)], ws, graph=False).run()


@pytest.mark.parametrize("batch,x_dtype", [(1, "f16"), (2, "f16"), (1, "f32")])
def test_grouped_launch_matches_single_calls(batch, x_dtype):
    """Independent GEMVs as one grouped launch (hqb_gemv_grouped, eager and captured): every
    call's outputs against its own launch within the FP32 contract (the grouped grid splits
    each call over fewer CTAs, so split-row sums may add in another order) and against FP64;
    repeated grouped launches give identical bytes."""
    import harpq_b200 as hqb
    from conftest import assert_close

    rng = np.random.default_rng(77 + batch)
    shapes = [(12288, 4096), (4096, 4096), (22016, 4096), (4096, 11008), (300, 520)]
    pms = [plane_matrix(random_matrix(rng, r, c, stages=2)) for r, c in shapes]
    tdt = torch.float16 if x_dtype == "f16" else torch.float32
    xs = [torch.from_numpy(rng.standard_normal((batch, c)).astype(np.float16)).cuda().to(tdt) for _, c in shapes]
    ys = [torch.empty(batch, r, dtype=torch.float32, device="cuda") for r, _ in shapes]
    xd = hqb.F16 if x_dtype == "f16" else hqb.F32
    ws = hqb.Workspace(max(pm.workspace_bytes(batch, xd) for pm in pms))
    calls = [(pm, x, 2, y, hqb.FLAG_PDL) for pm, x, y in zip(pms, xs, ys)]
    outs = []
    for graph in (False, True):
        step = hqb.Step(calls, ws, graph=graph, independent=True)
        for y in ys:
            y.fill_(float("nan"))
        step.run()
        torch.cuda.synchronize()
        outs.append([y.clone() for y in ys])
        step.close()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    for pm, x, y in zip(pms, xs, outs[0]):
        alone = pm.gemv(x, prefix=2, y_dtype=torch.float32, workspace=ws)
        assert_close(y.cpu().numpy(), alone.cpu().numpy(), 2e-4, 2e-4, "grouped vs alone")
        e64 = (x.double() @ pm.decode(2).double().T).cpu().numpy()
        assert_close(y.cpu().numpy(), e64, 2e-4, 2e-4, "grouped vs FP64")
    assert ws.error_flags() == 0


@pytest.mark.parametrize("independent", [False, True])
def test_step_with_captured_host_copies(independent):
    """hqb_step_create_io: the step's graph copies pinned host x in, runs the GEMVs and
    copies y out; each launch moves the host buffers' current contents."""
    import harpq_b200 as hqb

    rng = np.random.default_rng(77)
    shapes = [(768, 512), (1024, 1000), (300, 512)]
    pms = [plane_matrix(random_matrix(rng, r, c, stages=2)) for r, c in shapes]
    cols = [c for _, c in shapes]
    rows = [r for r, _ in shapes]
    x_all = torch.empty(sum(cols), dtype=torch.float16, device="cuda")
    y_all = torch.empty(sum(rows), dtype=torch.float16, device="cuda")
    xs, ys, o = [], [], 0
    for c in cols:
        xs.append(x_all[o:o + c].view(1, c))
        o += c
    o = 0
    for r in rows:
        ys.append(y_all[o:o + r].view(1, r))
        o += r
    hx = torch.empty(sum(cols), dtype=torch.float16).pin_memory()
    hy = torch.empty(sum(rows), dtype=torch.float16).pin_memory()
    ws = hqb.Workspace(max(pm.workspace_bytes(1, hqb.F16) for pm in pms))
    step = hqb.Step([(pm, x, 2, y, hqb.FLAG_PDL) for pm, x, y in zip(pms, xs, ys)], ws, independent=independent,
                    inputs=[(x_all, hx)], outputs=[(hy, y_all)])
    for trial in range(3):
        hx.copy_(torch.from_numpy(rng.standard_normal(sum(cols)).astype(np.float16)))
        hy.fill_(float("nan"))
        step.run()
        torch.cuda.synchronize()
        xd = hx.cuda()
        want, o = [], 0
        for pm, c in zip(pms, cols):
            want.append(pm.gemv(xd[o:o + c].view(1, c), prefix=2, y_dtype=torch.float16, workspace=ws))
            o += c
        assert torch.equal(hy, torch.cat(want, dim=1).view(-1).cpu()), f"trial {trial}"
    step.close()
    # host buffers 2 bytes past a 16-byte boundary: the copies fall back to cudaMemcpyAsync
    hx2 = torch.empty(sum(cols) + 8, dtype=torch.float16).pin_memory()[1:1 + sum(cols)]
    hy2 = torch.empty(sum(rows) + 8, dtype=torch.float16).pin_memory()[1:1 + sum(rows)]
    step = hqb.Step([(pm, x, 2, y, hqb.FLAG_PDL) for pm, x, y in zip(pms, xs, ys)], ws, independent=independent,
                    inputs=[(x_all, hx2)], outputs=[(hy2, y_all)])
    hx2.copy_(hx)
    hy2.fill_(float("nan"))
    step.run()
    torch.cuda.synchronize()
    assert torch.equal(hy2, hy)
    step.close()
    assert ws.error_flags() == 0
    # pageable host memory cannot sit in the graph
    with pytest.raises(ValueError):
        hqb.Step([(pms[0], xs[0], 2, ys[0], 0)], ws, inputs=[(x_all, torch.empty(sum(cols), dtype=torch.float16))])
