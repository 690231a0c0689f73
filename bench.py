"""Benchmark of the progressive int2 GEMV path on B200 (one JSON line on rank 0).

Workloads (seeded synthetic weights, FP16 activations):
  llama7b_block_p2   q,k,v,o 4096x4096; gate,up 11008x4096; down 4096x11008; prefix 2; 1 GPU
  llama70b_mlp_p3    gate,up 28672x8192; down 8192x28672; prefix 3; output rows sharded
                     over the ranks with an FP16 all-gather of each layer's output (NCCL)
Default: llama7b_block_p2 at one GPU, llama70b_mlp_p3 when --gpus > 1.  The single_*
workloads (one layer) serve profiling and per-shape checks.

A step is one pass over every layer of the workload at batch 1.  `value` is the
aggregate algorithmic HBM bytes (selected planes + scales + FP16 x + FP16 y, the
same bytes the reference's layout would need) per second over all ranks; weight
buffers rotate over copies totalling > 3x L2 so every step streams from HBM.

--impl reference times the reference's own C++ ProgressiveLinearReference
(native/src/stage_codec.cpp, compiled in place into oracle/_ref) on the host cores
for the same workload and metric.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "harp-q_b200"))

METRIC = "µs per layer & achieved HBM GB/s vs B200 peak, batch-1 GEMV at prefix depth 1–4"
L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    # name: (prefix, [(layer, rows, cols, input)], std, per-rank sharding)
    "llama7b_block_p2": (2, [("q", 4096, 4096, "a"), ("k", 4096, 4096, "a"), ("v", 4096, 4096, "a"),
                             ("o", 4096, 4096, "b"), ("gate", 11008, 4096, "c"), ("up", 11008, 4096, "c"),
                             ("down", 4096, 11008, "d")], 0.02),
    "llama70b_mlp_p3": (3, [("gate", 28672, 8192, "a"), ("up", 28672, 8192, "a"), ("down", 8192, 28672, "b")],
                        0.015),
    "single_4096_p1": (1, [("w", 4096, 4096, "a")], 0.02),
    "single_4096_p4": (4, [("w", 4096, 4096, "a")], 0.02),
    "single_11008_p1": (1, [("w", 11008, 4096, "a")], 0.02),
    "single_11008_p4": (4, [("w", 11008, 4096, "a")], 0.02),
    "single_28672_p1": (1, [("w", 28672, 8192, "a")], 0.015),
    "single_28672_p3": (3, [("w", 28672, 8192, "a")], 0.015),
}


def algorithmic_bytes(rows: int, cols: int, prefix: int, batch: int = 1) -> int:
    """d*17*N*K/64 (codes + one FP16 scale per row per 128 columns) + FP16 x and y."""
    return prefix * (rows * cols // 4 + rows * (-(-cols // 128)) * 2) + 2 * cols * batch + 2 * rows * batch


# ---------------------------------------------------------------------------------------
# synthetic weights: the reference's LS int2 fit (quantization.py:466-521) restated with
# torch on the GPU, for input generation only (never timed).  Same steps as
# oracle/quantize.py; FP64 reduction order may differ in the last bit.

def quantize_gpu(w: torch.Tensor, stages: int = 4):
    n, k = w.shape
    npad, kpad = -(-n // 128) * 128, -(-k // 128) * 128
    res = torch.zeros(npad, kpad, dtype=torch.float32, device=w.device)
    res[:n, :k] = w
    codes_out, bits_out = [], []
    for _ in range(stages):
        g = res.view(npad, kpad // 128, 128)
        peak = g.abs().amax(-1)
        s = torch.where(peak > 0, peak / 1.5, torch.zeros_like(peak))
        for _ in range(4):
            nz = (s != 0)[..., None]
            q = torch.where(nz, g / torch.where(nz, s[..., None], torch.ones_like(s[..., None])), torch.zeros_like(g))
            c = torch.clamp(torch.round(q), -2, 1)
            num = (g.double() * c.double()).sum(-1)
            den = (c.double() ** 2).sum(-1)
            fit = torch.where(den != 0, num / torch.where(den != 0, den, torch.ones_like(den)), torch.zeros_like(num))
            s = torch.where(den != 0, fit, s.double()).float().clamp_min(0.0)
        s16 = s.half()
        ex = s16.float()
        nz = (ex != 0)[..., None]
        q = torch.where(nz, g / torch.where(nz, ex[..., None], torch.ones_like(ex[..., None])), torch.zeros_like(g))
        c = torch.clamp(torch.round(q), -2, 1)
        res -= (c * ex[..., None]).view(npad, kpad)
        two = (c.to(torch.int8) & 3).to(torch.uint8).view(-1, 4)
        packed = two[:, 0] | (two[:, 1] << 2) | (two[:, 2] << 4) | (two[:, 3] << 6)
        codes_out.append(packed.contiguous())
        # scale layout [tile_row][tile_col][row_in_tile]
        bits = s16.view(npad // 128, 128, kpad // 128).permute(0, 2, 1).contiguous().view(-1).view(torch.int16)
        bits_out.append(bits)
        del g, q, c, two
    return codes_out, bits_out


def make_layer(rows, cols, std, seed, device):
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    w = torch.randn(rows, cols, generator=gen, device=device, dtype=torch.float32) * std
    codes, bits = quantize_gpu(w)
    del w
    return codes, bits


# ---------------------------------------------------------------------------------------
# clocks

class ClockSampler:
    """SM clock and clock-event reasons sampled through NVML (read-only queries) on a
    background thread every ~2 ms while the benchmark runs.  summary() reports the
    samples taken inside the timed region [t0, t1] (host monotonic time); when the
    region is too short for any sample it falls back to the whole measurement phase
    and says so in "window"."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.samples: list[tuple[float, int, int]] = []
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self._thread = None
        self.nv = None
        self.handle = None

    def _open(self):
        import pynvml as nv

        nv.nvmlInit()
        self.nv = nv
        handle = None
        try:
            props = torch.cuda.get_device_properties(self.device_index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            handle = nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:  # older torch without PCI ids: map through CUDA_VISIBLE_DEVICES
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            ids = [v.strip() for v in visible.split(",")] if visible else []
            idx = ids[self.device_index] if self.device_index < len(ids) else str(self.device_index)
            handle = (nv.nvmlDeviceGetHandleByUUID(idx) if not idx.isdigit()
                      else nv.nvmlDeviceGetHandleByIndex(int(idx)))
        self.handle = handle
        self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM)

    def _run(self):
        nv, h = self.nv, self.handle
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            except Exception as exc:  # keep the benchmark running; report the failure
                self.error = str(exc)
                return
            self.samples.append((time.monotonic(), mhz, reasons))
            self._stop.wait(0.002)

    def __enter__(self):
        try:
            self._open()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception as exc:
            self.error = str(exc)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)
        if self.nv is not None:
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass

    def summary(self, t0: float, t1: float) -> dict:
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        window = "timed region"
        if not inside:
            inside, window = self.samples, "measurement phase (timed region shorter than one sample)"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "error": self.error or "no samples"}
        reasons = set()
        for _, _, mask in inside:
            for name, attr in self.REASONS:
                if mask & getattr(self.nv, attr, 0):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(inside), "window": window,
                "sm_mhz_min": min(s[1] for s in inside)}


# ---------------------------------------------------------------------------------------
# our arm

def group_bytes(members, cols, prefix, batch=1):
    """Algorithmic bytes of one launch over row-stacked members sharing one input: the
    selected planes and scales of every member, the input once, every output."""
    rows = sum(m["nrows"] for m in members)
    return (prefix * (rows * cols // 4 + rows * (-(-cols // 128)) * 2) + 2 * cols * batch
            + 2 * rows * batch)


def build_workload(name, rank, world, device, rotation_target):
    """The workload's layers as launch groups.  Layers that share their input (q, k, v;
    gate, up) are row-stacked into one plane matrix and run as one GEMV launch, as a
    fused QKV / gate-up projection does; every other layer is its own launch."""
    import harpq_b200 as hqb

    prefix, layers, std = WORKLOADS[name]
    groups: dict = {}
    for li, (lname, rows, cols, src) in enumerate(layers):
        codes, bits = make_layer(rows, cols, std, 1000 + li, device)
        r0, nrows = (0, rows) if world == 1 else hqb.shard_rows(rows, world, rank)
        if world > 1:
            codes, bits = hqb.slice_stage_rows(codes, bits, cols, r0, nrows)
            codes = [c.contiguous() for c in codes]
            bits = [b.contiguous() for b in bits]
        pm = hqb.PlaneMatrix.from_stages(nrows, cols, codes, bits)
        del codes, bits
        g = groups.setdefault(src, {"src": src, "cols": cols, "members": [], "mats": []})
        g["members"].append({"name": lname, "rows": rows, "r0": r0, "nrows": nrows})
        g["mats"].append(pm)
    built = []
    for g in groups.values():
        mats = g.pop("mats")
        stacked = mats[0] if len(mats) == 1 else hqb.PlaneMatrix.stack(mats)
        del mats
        g["name"] = "+".join(m["name"] for m in g["members"])
        g["nrows"] = stacked.rows
        g["copies"] = [stacked]
        g["bytes"] = group_bytes(g["members"], g["cols"], prefix)
        # every rank gathers the same slot size: the largest stacked shard
        shard_rows = []
        for r in range(world):
            sizes = [hqb.shard_rows(m["rows"], world, r)[1] if world > 1 else m["rows"] for m in g["members"]]
            shard_rows.append(sum(-(-n // 128) * 128 for n in sizes[:-1]) + sizes[-1])
        g["slot_rows"] = max(shard_rows)
        built.append(g)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    step_bytes = sum(g["bytes"] for g in built)
    plane_bytes_step = sum(sum(p.numel() for p in g["copies"][0].planes[:prefix]) for g in built)
    ncopies = max(2, -(-rotation_target // max(1, plane_bytes_step)))
    ncopies += ncopies % 2  # consecutive steps alternate the two gathered-output buffers
    for g in built:
        base = g["copies"][0]
        for _ in range(ncopies - 1):
            cp = hqb.PlaneMatrix(base.rows, base.cols)
            cp.planes = [p.clone() for p in base.planes]
            g["copies"].append(cp)
    torch.cuda.synchronize()
    n_layers = len(layers)
    return prefix, built, step_bytes, ncopies, n_layers


def run_ours(args, rank, world, device):
    import harpq_b200 as hqb

    name = args.workload
    prefix, groups, step_bytes, ncopies, n_layers = build_workload(name, rank, world, device, 3 * L2_BYTES)
    srcs = {g["src"]: g["cols"] for g in groups}
    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    # every input of a step in one device buffer and every output in another (views per
    # group), so a step moves its inputs and outputs with one copy each way
    x_all = torch.empty(sum(srcs.values()), dtype=torch.float16, device=device)
    x_dev, off = {}, 0
    for s_, k in srcs.items():
        x_dev[s_] = x_all[off:off + k].view(1, k)
        x_dev[s_].copy_(torch.randn(1, k, generator=gen, device=device).half())
        off += k
    y_all = torch.empty(sum(g["nrows"] for g in groups), dtype=torch.float16, device=device)
    y_loc, off = {}, 0
    for g in groups:
        y_loc[g["name"]] = y_all[off:off + g["nrows"]].view(1, g["nrows"])
        off += g["nrows"]
    y_full = {g["name"]: torch.empty(world, g["slot_rows"], dtype=torch.float16, device=device) for g in groups}
    # N > 1: NCCL all_gather_into_tensor of each group's output slices; --fused-gather uses
    # the fused all-gather instead (outputs stored into every rank's buffer over NVLink by
    # the GEMV itself, then a bounded flag wait), two buffers per group alternating by step
    fused = world > 1 and args.fused_gather
    gathers = {g["name"]: [hqb.Gather(g["slot_rows"], 1, torch.float16) for _ in range(2)] for g in groups} \
        if fused else {}
    ws_bytes = max(g["copies"][0].workspace_bytes(1, hqb.F16) for g in groups)
    ws = hqb.Workspace(ws_bytes, device)
    # per step: the launches of each group's GEMV by the library's own dispatch rule (the
    # uniform kernel prepares its raw activations itself where they fit)
    launches_per_step = sum(g["copies"][0].gemv_launches(1, hqb.F16, prefix) + (1 if fused else 0) for g in groups)
    if world == 1 and args.step_mode == "grouped":
        launches_per_step = 1
    # N > 1, grouped: each group's shard output at a fixed offset of one padded buffer
    # (slot_rows per group), the step's GEMVs as one grouped launch per rank, then ONE NCCL
    # all-gather of the whole buffer
    mg_grouped = world > 1 and not fused and args.step_mode == "grouped"
    if mg_grouped:
        launches_per_step = 1
        slot_tot = sum(g["slot_rows"] for g in groups)
        y_pad_all = torch.zeros(slot_tot, dtype=torch.float16, device=device)
        y_pad, off = {}, 0
        for g in groups:
            y_pad[g["name"]] = y_pad_all[off:off + g["nrows"]].view(1, g["nrows"])
            off += g["slot_rows"]
        y_full_all = torch.empty(world, slot_tot, dtype=torch.float16, device=device)
        mg_steps = [hqb.Step([(G["copies"][c], x_dev[G["src"]], prefix, y_pad[G["name"]], hqb.FLAG_PDL)
                              for G in groups], ws, graph=False, independent=True) for c in range(ncopies)]

        def gather_all():
            torch.distributed.all_gather_into_tensor(y_full_all.view(-1), y_pad_all)

        def gstep(copy):
            mg_steps[copy].run()
            gather_all()

    def gather(g):
        if world == 1:
            return
        n = g["nrows"]
        pad = g["slot_rows"]
        send = y_loc[g["name"]] if n == pad else torch.nn.functional.pad(y_loc[g["name"]], (0, pad - n))
        torch.distributed.all_gather_into_tensor(y_full[g["name"]].view(-1), send.view(-1))

    def step(copy, x_src=None):
        xs = x_dev if x_src is None else x_src
        for g in groups:
            pm = g["copies"][copy]
            if fused:
                G = gathers[g["name"]][copy % 2]
                pm.gemv_gather(xs[g["src"]], G, prefix=prefix, workspace=ws, flags=hqb.FLAG_PDL)
            else:
                pm.gemv(xs[g["src"]], prefix=prefix, out=y_loc[g["name"]], workspace=ws, flags=hqb.FLAG_PDL)
                gather(g)
        # the workload's layers take given inputs, so each gathered output is waited for
        # once per step, before anything reads it (here: the end of the step)
        for g in groups:
            if fused:
                gathers[g["name"]][copy % 2].wait()

    # clocks are sampled from warm-up to the end of the e2e leg; the summary keeps the
    # samples that fall inside the timed region
    clk = ClockSampler(torch.cuda.current_device()).__enter__()

    # warm-up (also JIT/driver setup)
    for i in range(max(3, args.warmup)):
        step(i % ncopies)
    torch.cuda.synchronize()

    # one CUDA graph per weight copy; at N > 1 it includes the NCCL all-gathers
    use_graph = not args.no_graph
    graphs = []
    if use_graph:
        for c in range(ncopies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step(c)
            graphs.append(g)
        for i in range(3):
            graphs[i % ncopies].replay()
        torch.cuda.synchronize()

    ggraphs = []
    if mg_grouped:
        for i in range(max(3, args.warmup)):
            gstep(i % ncopies)
        torch.cuda.synchronize()
        for c in range(ncopies):
            g_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_):
                gstep(c)
            ggraphs.append(g_)
        for i in range(3):
            ggraphs[i % ncopies].replay()
        torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # ---- timed region: K steps, repeated; each repeat bracketed by a barrier and a
    # synchronize on both sides and timed with CUDA events, the max over ranks taken per
    # repeat; the headline is the median repeat
    repeats = max(1, args.repeats)

    def time_steps(run_one):
        out = []
        for _ in range(repeats):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            start.record()
            for i in range(args.steps):
                run_one(i)
            end.record()
            barrier()
            ms = start.elapsed_time(end)
            if world > 1:
                t = torch.tensor([ms], device=device)
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
                ms = float(t.item())
            out.append(ms / args.steps)
        return out

    # the step's GEMVs as one grouped launch (hqb_gemv_grouped: the workload's layers take
    # inputs of their own, so they are independent); N > 1: mg_grouped above
    grouped = world == 1 and args.step_mode == "grouped"
    gsteps = []
    if grouped:
        gsteps = [hqb.Step([(G["copies"][c], x_dev[G["src"]], prefix, y_loc[G["name"]], hqb.FLAG_PDL)
                            for G in groups], ws, graph=True, independent=True) for c in range(ncopies)]
        for i in range(3):
            gsteps[i % ncopies].run()
        torch.cuda.synchronize()
    t_timed0 = time.monotonic()
    chained_ms = time_steps(lambda i: graphs[i % ncopies].replay() if use_graph else step(i % ncopies))
    grouped_ms = time_steps(lambda i: gsteps[i % ncopies].run()) if grouped else None
    if mg_grouped:
        grouped_ms = time_steps(lambda i: ggraphs[i % ncopies].replay())
    t_timed1 = time.monotonic()
    rep_ms = grouped_ms if (grouped or mg_grouped) else chained_ms
    ms_per_step = statistics.median(rep_ms)
    # whole-job bytes: the full (unsharded) layers, each input once per group
    total_bytes = sum(group_bytes([{"nrows": m["rows"]} for m in g["members"]], g["cols"], prefix) for g in groups)
    value = total_bytes / (ms_per_step * 1e-3) / 1e9

    # ---- per-kernel roofline: each layer's GEMV launched back to back (PDL) inside one
    # CUDA graph over its rotating weight copies; CUDA events on the launching stream
    # around graph replays give the average duration of one launch
    kern = {}
    tot_b, tot_ms = 0, 0.0
    by_kernel = {}  # kernel name -> [algorithmic bytes, ms] over one launch per group
    per_graph = 4 * ncopies
    for G in groups:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(2):
                G["copies"][i % ncopies].gemv(x_dev[G["src"]], prefix=prefix, out=y_loc[G["name"]], workspace=ws,
                                              flags=hqb.FLAG_PDL)
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(g):
            for i in range(per_graph):
                G["copies"][i % ncopies].gemv(x_dev[G["src"]], prefix=prefix, out=y_loc[G["name"]], workspace=ws,
                                              flags=hqb.FLAG_PDL)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        per_launch_ms = e0.elapsed_time(e1) / (5 * per_graph)
        del g
        b = G["bytes"]
        kname = G["copies"][0].gemv_kernel(1, hqb.F16, prefix)
        kern[G["name"]] = {"us": round(per_launch_ms * 1e3, 3), "gbs": round(b / (per_launch_ms * 1e-3) / 1e9, 1),
                           "rows": G["nrows"], "cols": G["cols"], "kernel": kname}
        by_kernel.setdefault(kname, [0, 0.0])
        by_kernel[kname][0] += b
        by_kernel[kname][1] += per_launch_ms
        tot_b += b
        tot_ms += per_launch_ms
    if grouped:
        # one kernel per step: its launches back to back (the grouped step graph) are the step
        by_kernel = {"gemv_grouped_kernel": [sum(G["bytes"] for G in groups), ms_per_step]}
        tot_ms = ms_per_step
    mg_gemv_ms = None
    if mg_grouped:
        # this rank's grouped launch alone (graph of back-to-back launches, no gather)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(2):
                mg_steps[i % ncopies].run()
        torch.cuda.current_stream().wait_stream(side)
        gq = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gq):
            for i in range(per_graph):
                mg_steps[i % ncopies].run()
        for _ in range(3):
            gq.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            gq.replay()
        e1.record()
        torch.cuda.synchronize()
        mg_gemv_ms = e0.elapsed_time(e1) / (5 * per_graph)
        del gq
        by_kernel = {"gemv_grouped_kernel": [sum(G["bytes"] for G in groups), mg_gemv_ms]}
        tot_ms = mg_gemv_ms
    # the roofline line is the kernel with the most device time; every kernel's share is listed
    dominant = max(by_kernel, key=lambda k: by_kernel[k][1])
    dom_b, dom_ms = by_kernel[dominant]
    achieved = dom_b / (dom_ms * 1e-3) / 1e9

    # ---- N > 1: the step's collective alone (the NCCL all-gathers of every group, in one
    # graph), so that the step splits into per-rank GEMV time and gather time
    gather_us = None
    if world > 1 and not fused:
        gg = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            if mg_grouped:
                gather_all()
            else:
                for G in groups:
                    gather(G)
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(gg):
            for _ in range(8):
                if mg_grouped:
                    gather_all()
                else:
                    for G in groups:
                        gather(G)
        for _ in range(2):
            gg.replay()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            gg.replay()
        e1.record()
        barrier()
        t = torch.tensor([e0.elapsed_time(e1) / 40.0], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        gather_us = round(float(t.item()) * 1e3, 3)
        del gg
    gemv_us = sum(v["us"] for v in kern.values()) if mg_gemv_ms is None else mg_gemv_ms * 1e3
    if world > 1:
        t = torch.tensor([gemv_us], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        gemv_us = float(t.item())

    # ---- e2e through the public API: pinned host x -> device, GEMVs, device -> host y.
    # One host->device copy of the step's inputs and one device->host copy of its outputs
    # every step; at N = 1 copies and GEMVs are one library step (hqb.Step with inputs and
    # outputs), at N > 1 call by call with the all-gathers between them.
    host_x_all = x_all.cpu().pin_memory()

    def gathered(g, copy):
        if fused:
            return gathers[g["name"]][copy % 2].out
        return y_full[g["name"]] if world > 1 else y_loc[g["name"]]

    if mg_grouped:
        host_y = {"all": torch.empty_like(y_full_all, device="cpu").pin_memory()}
    elif world == 1:
        # each step is one hqb.Step whose graph holds the input copy, the GEMVs and the
        # output copy (hqb_step_create_io); one host call per step
        host_y_all = torch.empty_like(y_all, device="cpu").pin_memory()
        steps_api = [hqb.Step([(G["copies"][c], x_dev[G["src"]], prefix, y_loc[G["name"]], hqb.FLAG_PDL)
                               for G in groups], ws, independent=grouped, inputs=[(x_all, host_x_all)],
                              outputs=[(host_y_all, y_all)]) for c in range(ncopies)]
        host_y = {"all": host_y_all}
    else:
        host_y = {g["name"]: torch.empty_like(gathered(g, 0), device="cpu").pin_memory() for g in groups}

    def e2e_step(copy):
        if mg_grouped:
            x_all.copy_(host_x_all, non_blocking=True)
            ggraphs[copy].replay()
            host_y["all"].copy_(y_full_all, non_blocking=True)
        elif world == 1:
            steps_api[copy].run()
        else:
            x_all.copy_(host_x_all, non_blocking=True)
            step(copy)
            for g in groups:
                host_y[g["name"]].copy_(gathered(g, copy), non_blocking=True)

    for i in range(3):
        e2e_step(i % ncopies)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        e2e_step(i % ncopies)
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_ms /= args.steps
    h2d = host_x_all.numel() * 2
    d2h = sum(y.numel() * 2 for y in host_y.values())

    clk.__exit__(None, None, None)
    del graphs, ggraphs  # graphs holding NCCL work are released before the process group is destroyed
    torch.cuda.synchronize()
    gather_flags = 0
    for pair in gathers.values():
        for G in pair:
            gather_flags |= int(G.device_flags.item())
    if world > 1:
        torch.distributed.barrier()  # every rank is done with the peers' buffers
    for pair in gathers.values():
        for G in pair:
            G.close()
    flags = ws.error_flags()
    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "us_per_layer": round(ms_per_step * 1e3 / n_layers, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int2 codes x FP16 scales, FP16 x/y, FP32 accumulate",
        "data": "synthetic: seeded N(0,std) weights quantized by the reference LS int2 fit (GPU restatement), "
                "seeded N(0,1) FP16 activations",
        "config": {"workload": name, "prefix": prefix, "batch": 1,
                   "layers": [[m["name"], m["rows"], g["cols"]] for g in groups for m in g["members"]],
                   "launches": [[g["name"], g["nrows"], g["cols"]] for g in groups],
                   "grouping": "layers sharing an input run as one row-stacked launch; step_mode grouped: "
                               "the launch groups (independent inputs) run as one grouped kernel launch, "
                               "at N > 1 followed by one all-gather of every group's output",
                   "parallelism": (f"row-shard{world}+" + ("fused-p2p-allgather" if fused else
                                                            "one-nccl-allgather-per-step" if mg_grouped else
                                                            "nccl-allgather-per-group"))
                                  if world > 1 else "single",
                   "l2": f"{ncopies} rotating weight copies, {ncopies * step_bytes / 2**20:.0f} MiB > 3x L2",
                   "graph": use_graph},
        "roofline": None,
        "kernels": kern,
        "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "us_per_step": round(e2e_ms * 1e3, 2), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps * repeats,
        "timing": {"repeats": repeats, "steps_per_repeat": args.steps,
                   "ms_per_step": [round(v, 5) for v in rep_ms], "median_ms": round(ms_per_step, 5),
                   "min_ms": round(min(rep_ms), 5), "max_ms": round(max(rep_ms), 5)},
        "step_mode": "grouped" if (grouped or mg_grouped) else "chained",
        # the same step as dependent launches (one launch per layer group, PDL between them,
        # as a decoder block whose layers wait for each other runs)
        "chained": {"value": round(total_bytes / (statistics.median(chained_ms) * 1e-3) / 1e9, 1),
                    "ms_per_step": round(statistics.median(chained_ms), 5),
                    "launches_per_step": sum(g["copies"][0].gemv_launches(1, hqb.F16, prefix) for g in groups)},
        "clocks": clk.summary(t_timed0, t_timed1),
        "device_error_flags": flags | gather_flags,
    }
    if world > 1:
        # per rank (max over ranks): the GEMV launches of a step timed alone, the step's
        # gather alone (NCCL; the fused gather stores inside the GEMV), and the whole step
        result["per_rank"] = {"gemv_us": round(gemv_us, 3), "gather_us": gather_us,
                              "step_us": round(ms_per_step * 1e3, 3),
                              "gather": "fused-p2p" if fused else
                                        ("one nccl all_gather_into_tensor of every group's output" if mg_grouped
                                         else "nccl all_gather_into_tensor per group")}
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    peak = peaks.get("hbm_gbs", 6650.0)
    traffic = _recorded_traffic_ratio()
    result["roofline"] = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                          "frac": round(achieved / peak, 4),
                          "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                          "traffic": None if traffic is None else round(traffic * dom_b / max(1, len(
                              [g for g in kern.values() if g["kernel"] == dominant]))),
                          "kernel": f"hqb::{dominant} (activation preparation and split-row sums inside)",
                          "achieved_note": "algorithmic bytes of one launch per group run by this kernel / sum of "
                                           "those groups' average launch durations (CUDA events around graphs of "
                                           "back-to-back launches)",
                          "by_kernel": {k: {"achieved": round(v[0] / (v[1] * 1e-3) / 1e9, 1),
                                            "frac": round(v[0] / (v[1] * 1e-3) / 1e9 / peak, 4),
                                            "time_share": round(v[1] / tot_ms, 3)}
                                        for k, v in by_kernel.items()}}
    return result


def _recorded_traffic_ratio():
    """DRAM bytes per algorithmic byte of the GEMV kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "gemv_kernel_traffic.txt"
    try:
        for line in p.read_text().splitlines():
            if line.startswith("dram_bytes_per_algorithmic_byte:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------------------
# supplementary single-GPU measurements (BASELINE configs 4 and 5, and the sharded
# workload at one GPU); weights are random codes and scales: timing does not depend on
# their values

def _random_plane_matrix(rows, cols, gen, device):
    import harpq_b200 as hqb

    g = hqb.geometry(rows, cols)
    codes, bits = [], []
    for _ in range(4):
        codes.append(torch.randint(0, 256, (g.padded_rows * g.padded_columns // 4,), dtype=torch.uint8,
                                   device=device, generator=gen))
        sc = (torch.rand(g.padded_rows // 128 * (g.padded_columns // 128) * 128, device=device, generator=gen)
              * 0.01 + 1e-3).half()
        bits.append(sc.view(torch.int16))
    return hqb.PlaneMatrix.from_stages(rows, cols, codes, bits)


def _graph_us(fn, launches, reps=5):
    """Average µs per call of fn(i) over a CUDA graph of `launches` calls."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for i in range(2):
            fn(i)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(launches):
            fn(i)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / (reps * launches)


def supplementary(device):
    import harpq_b200 as hqb

    gen = torch.Generator(device=device)
    gen.manual_seed(11)
    out = {}
    # config 4: mixed depth, 11008x4096, per-tile depth uniform in {1..4} (seed 7), batch 1
    copies = [_random_plane_matrix(11008, 4096, gen, device) for _ in range(4)]
    gr, gc = copies[0].grid_rows, copies[0].grid_cols
    depth = torch.from_numpy(np.random.default_rng(7).integers(1, 5, size=(gr, gc)).astype(np.uint8)).to(device)
    plan = hqb.DepthPlan(depth, 4)
    x = torch.randn(1, 4096, device=device, generator=gen).half()
    y = torch.empty(1, 11008, device=device, dtype=torch.float16)
    ws = hqb.Workspace(copies[0].workspace_bytes(16, hqb.F16), device)
    mixed_bytes = int(depth.sum().item()) * 4352 + 2 * 4096 + 2 * 11008
    us = _graph_us(lambda i: copies[i % 4].gemv(x, depth=plan, out=y, workspace=ws, flags=hqb.FLAG_PDL), 32)
    uni = {p: _graph_us(lambda i: copies[i % 4].gemv(x, prefix=p, out=y, workspace=ws, flags=hqb.FLAG_PDL), 32)
           for p in (2, 3)}
    out["mixed_depth_11008x4096"] = {"us": round(us, 3), "gbs": round(mixed_bytes / (us * 1e-6) / 1e9, 1),
                                     "mean_depth": round(mixed_bytes / (gr * gc * 4352), 3),
                                     "uniform_p2_us": round(uni[2], 3), "uniform_p3_us": round(uni[3], 3)}
    # config 5: small batch at prefix 4, tensor-core kernel vs the CUDA-core comparison kernel
    sb = {}
    for rows in (4096, 11008):
        mats = copies if rows == 11008 else [_random_plane_matrix(4096, 4096, gen, device) for _ in range(4)]
        for batch in (2, 4, 8, 16):
            xb = torch.randn(batch, 4096, device=device, generator=gen).half()
            yb = torch.empty(batch, rows, device=device, dtype=torch.float16)
            nbytes = 4 * 17 * rows * 4096 // 64 + 2 * 4096 * batch + 2 * rows * batch
            flops = 2.0 * batch * rows * 4096 * 4
            t = _graph_us(lambda i: mats[i % 4].gemv(xb, prefix=4, out=yb, workspace=ws, flags=hqb.FLAG_PDL), 32)
            e = {"tensor_us": round(t, 3), "tensor_gbs": round(nbytes / (t * 1e-6) / 1e9, 1),
                 "tensor_tflops": round(flops / (t * 1e-6) / 1e12, 2)}
            if batch <= 8:
                t2 = _graph_us(lambda i: mats[i % 4].gemv(xb, prefix=4, out=yb, workspace=ws,
                                                          flags=hqb.FLAG_SIMT), 32)
                e.update({"simt_us": round(t2, 3), "simt_gbs": round(nbytes / (t2 * 1e-6) / 1e9, 1)})
            sb[f"{rows}x4096_b{batch}"] = e
        del mats
    out["small_batch_p4"] = sb
    # prefill (hqb_prefill_gemm): FP16 decode of the selected stages + cuBLAS FP16 GEMM,
    # 11008x4096 at prefix 2, weights rotating; the GEMV at batch 16 beside it
    pw = torch.empty(copies[0].prefill_workspace_bytes(), dtype=torch.uint8, device=device)
    pf = {}
    for batch in (16, 64, 256, 1024):
        xb = torch.randn(batch, 4096, device=device, generator=gen).half()
        yb = torch.empty(batch, 11008, device=device, dtype=torch.float16)
        t = _graph_us(lambda i: copies[i % 4].prefill(xb, 2, out=yb, workspace=pw), 8)
        e = {"us": round(t, 3), "tflops": round(2.0 * batch * 11008 * 4096 / (t * 1e-6) / 1e12, 1)}
        if batch == 16:
            tg = _graph_us(lambda i: copies[i % 4].gemv(xb, prefix=2, out=yb, workspace=ws, flags=hqb.FLAG_PDL), 32)
            e["gemv_us"] = round(tg, 3)
        pf[f"11008x4096_p2_b{batch}"] = e
    out["prefill"] = pf
    del pw, copies
    torch.cuda.empty_cache()
    out["prefix_sweep"] = prefix_sweep(device, gen)
    out["reference_gpu_kernel"] = reference_gpu_kernel(device, gen)
    return out


def prefix_sweep(device, gen):
    """The metric at every prefix depth: config 1 (4096x4096) and the 7B MLP shapes
    (11008x4096, 4096x11008), batch 1, FP16 x/y, the library's default kernel per shape;
    weights rotate over > 3x L2."""
    import harpq_b200 as hqb

    res = {}
    for rows, cols in ((4096, 4096), (11008, 4096), (4096, 11008)):
        per_copy = 4 * 17 * rows * cols // 64
        n = max(2, -(-3 * L2_BYTES // per_copy))
        mats = [_random_plane_matrix(rows, cols, gen, device) for _ in range(n)]
        x = torch.randn(1, cols, device=device, generator=gen).half()
        y = torch.empty(1, rows, device=device, dtype=torch.float16)
        ws = hqb.Workspace(mats[0].workspace_bytes(1, hqb.F16), device)
        for p in (1, 2, 3, 4):
            us = _graph_us(lambda i: mats[i % n].gemv(x, prefix=p, out=y, workspace=ws, flags=hqb.FLAG_PDL), 32)
            b = algorithmic_bytes(rows, cols, p)
            res[f"{rows}x{cols}_p{p}"] = {"us": round(us, 3), "gbs": round(b / (us * 1e-6) / 1e9, 1),
                                          "kernel": mats[0].gemv_kernel(1, hqb.F16, p)}
        del mats
        torch.cuda.empty_cache()
    return res


def reference_gpu_kernel(device, gen):
    """The reference's own ProgressiveGemvKernel (native/src/progressive_gemv.cu:348-411),
    compiled for sm_100a from its sources into oracle/_ref/libharpq_ref_gpu.so and launched
    through its LaunchProgressiveGemv, timed on this GPU next to this library's drop-in
    reference-layout kernels (hqb_raw_gemv: raw_i8_kernel by default, the per-element
    raw_gemv_kernel with HQB_RAW_GENERIC) and its plane kernel, on the same codes and scales
    (reference layout: row-major codes, FP16 scales), FP32 x/y as the reference takes them,
    weights rotating over > 3x L2."""
    import ctypes

    import harpq_b200 as hqb

    path = ROOT / "oracle" / "_ref" / "libharpq_ref_gpu.so"
    if not path.exists():
        return {"unavailable": "oracle/_ref/libharpq_ref_gpu.so not built"}
    R = ctypes.CDLL(str(path))
    R.hqr_gpu_launch.restype = ctypes.c_int
    R.hqr_gpu_launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                 ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    res = {}
    for rows, cols, p in ((4096, 4096, 2), (11008, 4096, 2)):
        g = hqb.geometry(rows, cols)
        per_copy = p * 17 * rows * cols // 64
        n = max(2, -(-3 * L2_BYTES // per_copy))
        raw = []
        for _ in range(n):
            codes = [torch.randint(0, 256, (g.padded_rows * g.padded_columns // 4,), dtype=torch.uint8, device=device,
                                   generator=gen) for _ in range(p)]
            bits = [(torch.rand(g.padded_rows // 128 * (g.padded_columns // 128) * 128, device=device, generator=gen)
                     * 0.01 + 1e-3).half().view(torch.int16) for _ in range(p)]
            raw.append((codes, bits))
        x = torch.randn(cols, device=device, generator=gen)
        y = torch.empty(rows, device=device)
        geo = (ctypes.c_uint64 * 7)(g.original_rows, g.original_columns, g.padded_rows, g.padded_columns,
                                    g.tile_rows, g.tile_columns, g.group_size)
        ptrs = [((ctypes.c_void_p * p)(*[c.data_ptr() for c in codes]), (ctypes.c_void_p * p)(*[b.data_ptr() for b in bits]))
                for codes, bits in raw]
        stream = lambda: torch.cuda.current_stream().cuda_stream

        def ref(i):
            rc = R.hqr_gpu_launch(geo, ptrs[i % n][0], ptrs[i % n][1], p, p, x.data_ptr(), None, y.data_ptr(), stream())
            if rc != 0:
                raise RuntimeError(f"reference LaunchProgressiveGemv: {rc}")

        mats = [hqb.RawMatrix(g, codes, bits) for codes, bits in raw]
        planes = [hqb.PlaneMatrix.from_stages(rows, cols, codes, bits) for codes, bits in raw]
        ws = hqb.Workspace(planes[0].workspace_bytes(1, hqb.F32), device)
        b = p * (rows * cols // 4 + rows * (cols // 128) * 2) + 4 * cols + 4 * rows  # FP32 x and y
        t_ref = _graph_us(ref, 16)
        t_raw = _graph_us(lambda i: mats[i % n].gemv(x, p, out=y, flags=hqb.RAW_REQUIRE_FAST), 16)
        t_generic = _graph_us(lambda i: mats[i % n].gemv(x, p, out=y, flags=hqb.RAW_GENERIC), 16)
        xr = x.view(1, -1)
        t_plane = _graph_us(lambda i: planes[i % n].gemv(xr, prefix=p, out=y.view(1, -1), workspace=ws,
                                                          flags=hqb.FLAG_PDL), 16)
        res[f"{rows}x{cols}_p{p}"] = {
            "reference_kernel_us": round(t_ref, 3), "reference_kernel_gbs": round(b / (t_ref * 1e-6) / 1e9, 1),
            "hqb_raw_gemv_us": round(t_raw, 3), "hqb_raw_gemv_gbs": round(b / (t_raw * 1e-6) / 1e9, 1),
            "hqb_raw_gemv_kernel": "raw_i8_kernel",
            "hqb_raw_generic_us": round(t_generic, 3),
            "hqb_raw_generic_gbs": round(b / (t_generic * 1e-6) / 1e9, 1),
            "raw_speedup_vs_reference_kernel": round(t_ref / t_raw, 2),
            "plane_us": round(t_plane, 3), "plane_gbs": round(b / (t_plane * 1e-6) / 1e9, 1),
            "plane_speedup_vs_reference_kernel": round(t_ref / t_plane, 2)}
        del raw, mats, planes, ptrs
        torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------------------
# reference arm / CPU baseline

def reference_inputs(name, device):
    """Host progressive matrices (oracle.Matrix) for the workload plus FP16-exact x."""
    from oracle import oracle as orc

    prefix, layers, std = WORKLOADS[name]
    mats, xs = [], {}
    for li, (lname, rows, cols, src) in enumerate(layers):
        if device is not None:
            codes, bits = make_layer(rows, cols, std, 1000 + li, device)
            codes = [c.cpu().numpy() for c in codes]
            scales = [b.cpu().numpy().view(np.float16).astype(np.float32) for b in bits]
        else:
            from oracle import quantize as qz
            rng = np.random.default_rng(1000 + li)
            q = qz.quantize(rng.normal(0, std, size=(rows, cols)).astype(np.float32))
            codes = q.codes
            scales = [s.astype(np.float32).reshape(-1) for s in q.scales]
        rp, cp = -(-rows // 128) * 128, -(-cols // 128) * 128
        mats.append((lname, src, orc.Matrix((rows, cols, rp, cp, 128, 128, 128), codes, scales)))
        xs.setdefault(src, np.random.default_rng(7).standard_normal(cols).astype(np.float16).astype(np.float32))
    return prefix, mats, xs


def time_reference(name, steps, warmup, device, threads=None, budget_s=None):
    from oracle import refcpu

    if not refcpu.available():
        raise RuntimeError("oracle/_ref/libharpq_ref.so is not built")
    threads = threads or os.cpu_count() or 1
    prefix, mats, xs = reference_inputs(name, device)
    runners = [(lname, src, m, refcpu.ShardedReference(m, threads)) for lname, src, m in mats]
    by_src: dict = {}
    for _, src, m, _ in runners:
        by_src.setdefault(src, (m.cols, []))[1].append({"nrows": m.rows})
    step_bytes = sum(group_bytes(members, cols, prefix) for cols, members in by_src.values())

    def one():
        for _, src, _, r in runners:
            r.linear(xs[src], prefix)

    for _ in range(warmup):
        one()
    times = []
    t_all = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        if budget_s is not None and time.perf_counter() - t_all > budget_s:
            break
    for *_, r in runners:
        r.close()
    mean = sum(times) / len(times)
    return {"value": round(step_bytes / mean / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"{len(times)} full {name} step(s), tile-row shards over {threads} threads, "
                      f"{mean * 1e3:.1f} ms/step", "ms_per_step": mean * 1e3, "steps_timed": len(times)}


def time_numpy_reference(name, device, budget_s=12.0):
    """The reference's NumPy progressive_matmul (src/harpq/quantization.py:352-406, restated
    in oracle/oracle.py: progressive_matmul_np) on the host: per layer, each selected stage
    decoded to dense FP32 and multiplied through BLAS with every host core.  Steps run until
    the budget is spent (at least one)."""
    from oracle import oracle as orc

    prefix, mats, xs = reference_inputs(name, device)
    by_src: dict = {}
    for _, src, m in mats:
        by_src.setdefault(src, (m.cols, []))[1].append({"nrows": m.rows})
    step_bytes = sum(group_bytes(members, cols, prefix) for cols, members in by_src.values())
    times = []
    t_all = time.perf_counter()
    while not times or (time.perf_counter() - t_all < budget_s and len(times) < 20):
        t0 = time.perf_counter()
        for _, src, m in mats:
            orc.progressive_matmul_np(m, xs[src], prefix)
        times.append(time.perf_counter() - t0)
    mean = sum(times) / len(times)
    blas = {k: os.environ[k] for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS") if k in os.environ}
    return {"value": round(step_bytes / mean / 1e9, 4), "unit": "GB/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{len(times)} full {name} step(s) of the NumPy progressive_matmul restatement, BLAS threads "
                      f"{blas or 'default (all cores)'}, {mean * 1e3:.1f} ms/step"}


def run_reference_arm(args, device):
    name = args.workload
    # each step is one full pass of the workload on the host cores; the run stops
    # after the step that crosses 60 s so that it ends within a few minutes
    r = time_reference(name, args.steps, max(1, min(args.warmup, 2)), device, budget_s=60.0)
    prefix, layers, _ = WORKLOADS[name]
    return {"metric": METRIC, "impl": "reference", "value": r["value"], "unit": "GB/s", "n_gpus": args.gpus,
            "steps": r["steps_timed"], "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 3),
            "us_per_layer": round(r["ms_per_step"] * 1e3 / len(layers), 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int2 codes x FP32 scales, FP32 x/y (reference C++)",
            "data": "synthetic, the product arm's weights (same seeds and quantizer)",
            "config": {"workload": name, "prefix": prefix, "batch": 1},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------------------

def profile_steps(args, device) -> int:
    """The workload's grouped step run eagerly args.ncu_steps times (hqb_gemv_grouped, one
    launch per step, rotating weight copies): a short, plain command for a profiler to
    capture (`ncu -k regex:gemv_grouped -s <warm-up> -c 1 python bench.py --ncu-steps 6`)."""
    import harpq_b200 as hqb

    prefix, groups, _, ncopies, _ = build_workload(args.workload, 0, 1, device, 3 * L2_BYTES)
    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    xs = {g["src"]: torch.randn(1, g["cols"], generator=gen, device=device).half() for g in groups}
    ys = {g["name"]: torch.empty(1, g["nrows"], dtype=torch.float16, device=device) for g in groups}
    ws = hqb.Workspace(max(g["copies"][0].workspace_bytes(1, hqb.F16) for g in groups), device)
    steps = [hqb.Step([(G["copies"][c], xs[G["src"]], prefix, ys[G["name"]], hqb.FLAG_PDL) for G in groups], ws,
                      graph=False, independent=True) for c in range(ncopies)]
    for i in range(args.ncu_steps):
        steps[i % ncopies].run()
    torch.cuda.synchronize()
    print(f"{args.ncu_steps} grouped steps of {args.workload}; device error flags {ws.error_flags()}")
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="auto", choices=["auto", *WORKLOADS])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the supplementary single-GPU measurements")
    ap.add_argument("--repeats", type=int, default=5, help="timed regions of --steps steps (median reported)")
    ap.add_argument("--step-mode", choices=["grouped", "chained"], default="grouped",
                    help="N = 1: the step's independent GEMVs as one grouped launch, or one launch per group")
    ap.add_argument("--fused-gather", action="store_true",
                    help="N > 1: gather outputs with the fused P2P gather instead of NCCL all_gather_into_tensor")
    ap.add_argument("--ncu-steps", type=int, default=0,
                    help="N = 1, for profiler captures: build the workload, run this many grouped steps "
                         "eagerly (no graph, no timing, no JSON line) and exit")
    args = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload == "auto":
        args.workload = "llama7b_block_p2" if world == 1 else "llama70b_mlp_p3"
    have_gpu = torch.cuda.is_available()
    device = torch.device("cuda", local) if have_gpu else None
    if have_gpu:
        torch.cuda.set_device(device)

    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference_arm(args, device)), flush=True)
        return 0

    if world > 1:
        import datetime

        # NCCL's own lines (banner, NCCL_DEBUG=INFO communicator lines) go to stdout before
        # the one JSON line, which rank 0 prints last
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    import harpq_b200  # noqa: F401  (fails loudly when the library is missing)

    if args.ncu_steps > 0:
        return profile_steps(args, device)
    result = run_ours(args, rank, world, device)
    if rank == 0 and world == 1 and not args.no_extras:
        result["supplementary"] = supplementary(device)
        if args.workload == "llama7b_block_p2":
            # the sharded workload at one GPU, the N=1 point of the multi-GPU series
            sub = argparse.Namespace(**{**vars(args), "workload": "llama70b_mlp_p3", "steps": min(args.steps, 200)})
            r70 = run_ours(sub, rank, world, device)
            result["supplementary"]["llama70b_mlp_p3_n1"] = {k: r70[k] for k in ("value", "unit", "ms_per_step")}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = time_reference(args.workload, 3, 1, device, budget_s=20.0)
        result["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        result["cpu_baseline"]["numpy"] = time_numpy_reference(args.workload, device)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
