"""Benchmark of the small-M projection on B200 (the decode configuration at N=1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mbp|reference]

Workload (one STEP): one call of each decode-GEMV shape -- fused QKV+gate (K=6144,
N=14336) and O (K=N=6144) at M in {1, 8, 16, 32} -- with plain N(0, 0.02) weights and with the 1%-x256 escape
variant: 16 calls.  The calls are ordered M-major over the four matrices (qkv, o, qkv-escape, o-escape), so
between two uses of one matrix at least 250 MB of other weights stream through the 126 MB L2: every call
reads its weights cold (inputs larger than L2; no flush kernel).  The step is captured once as a CUDA graph and
replayed (the reference's judge also timed graph replays).

value      = packed weight bytes of a step / device time of a step (TB/s): the headline metric's bandwidth
             form; per-shape us/call (graph replay over rotating copies of that matrix) are under "shapes".
e2e        = the same step through the public API (mbp.kernel_fn) from pinned host buffers: H2D of x, the call
             (new output tensor each call), D2H of the output, all inside the timed region.
roofline   = the QKV+gate GEMV launches against the measured HBM copy bandwidth (MEASURED_PEAKS.json).

--impl reference: the reference path's CPU implementation -- this build's C port of the oracle (decode +
FP32 accumulate), all host threads -- on a bounded row sample of the same 16 calls, rank 0 only.
Multi-GPU (torchrun, N > 1): the same step with every projection tensor-parallel over the N ranks (QKV+gate
column-parallel + all-gather, O row-parallel + all-reduce, exchanged by the GEMV's peer stores over NVLink;
`--transport nccl` for NCCL collectives): total work fixed ("strong" scaling), device time = max over ranks.
--ref-shapes: kernel_fn at the reference's 30 published (M, layer) shapes against its H200 numbers (one JSON
line, not the bench line).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "muse-bf16-proj_b200"))
sys.path.insert(0, ROOT)

METRIC = "µs/call cold-L2 & packed-weight HBM TB/s vs 8 TB/s peak, M=1–256"
SHAPES = {"qkv_gate": (14336, 6144), "o": (6144, 6144)}
MS = (1, 8, 16, 32)
MATS = (("qkv_gate", "plain"), ("o", "plain"), ("qkv_gate", "esc1pct"), ("o", "esc1pct"))
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one QKV+gate M=1 launch, from one ncu capture
NCU_TRAFFIC_QKV_M1 = 136081664


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def make_weight(n, k, variant, device):
    import torch
    torch.manual_seed(0)
    w = torch.randn(n, k) * 0.02
    if variant == "esc1pct":
        idx = torch.randperm(n * k, generator=torch.Generator().manual_seed(2))[: n * k // 100]
        w.view(-1)[idx] *= 256
    return w.to(torch.bfloat16).to(device)


def make_x(m, k, device):
    import torch
    g = torch.Generator().manual_seed(1)
    return torch.randn(m, k, generator=g).to(torch.bfloat16).to(device)


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.2)
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
        self.f.flush()
        self.f.seek(0)
        rows = [r.strip().split(", ") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, smax, reasons = [], None, set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                for nm, v in zip(self.FIELDS, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_run(steps: int, warmup: int, sample_rows: int):
    """The reference path on the host: the oracle's C port (decode + FP32 accumulate) over all host threads on a
    bounded row sample of every call.  Returns (TB/s of packed weights, seconds per sampled step, cores, text)."""
    import numpy as np
    import torch
    from oracle import oracle
    cores = os.cpu_count() or 1
    work, packed = [], {}
    for m in MS:
        for layer, variant in MATS:
            n, k = SHAPES[layer]
            if (layer, variant) not in packed:  # the packed sample does not depend on M
                w = make_weight(n, k, variant, "cpu")[:sample_rows]
                packed[layer, variant] = oracle.pack(w.view(torch.int16).numpy().view(np.uint16), tile_base=True)
            p = packed[layer, variant]
            x = make_x(m, k, "cpu").view(torch.int16).numpy().view(np.uint16)
            work.append((p, x, p["units"].nbytes + p["esc"].nbytes))
    for _ in range(warmup):
        for p, x, _b in work:
            oracle.gemv_packed(x, p, threads=cores)
    t0 = time.perf_counter()
    for _ in range(steps):
        for p, x, _b in work:
            oracle.gemv_packed(x, p, threads=cores)
    dt = (time.perf_counter() - t0) / max(steps, 1)
    nbytes = sum(b for _, _, b in work)
    return nbytes / dt / 1e12, dt, cores, f"first {sample_rows} rows of each of the {len(work)} calls of a step"


def run_reference(args, rank, world):
    if rank != 0:
        return
    # exactly --steps timed and --warmup untimed steps; each step is a row sample of the 16 calls (~55 ms for
    # 1024 rows on 16 cores), shrunk so that the whole run stays near a minute
    steps, warm = max(1, args.steps), max(0, args.warmup)
    rows = 1024
    while rows > 16 and (steps + warm) * rows * 55e-3 / 1024 > 60.0:
        rows //= 2
    v, dt, cores, sample = cpu_reference_run(steps, warm, sample_rows=rows)
    line = {"metric": METRIC, "value": round(v, 6), "unit": "TB/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warm, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (BASELINE.json config 2 recipe)",
            "config": {"workload": "config2 decode GEMV: qkv_gate 6144->14336 and o 6144->6144, M in {1,8,16,32}, "
                                   "plain + 1% x256 escape weights (16 calls per step)", "l2": "n/a (host)"},
            "impl": "reference",
            "cpu_baseline": {"value": round(v, 6), "unit": "TB/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 6), "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def graph_of(fn, stream):
    import torch
    fn()  # first call on the device: attributes, planning
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            fn()
    torch.cuda.synchronize()
    return g


def run_mbp(args, rank, world):
    import torch
    import torch.distributed as dist
    import mbp

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    side = torch.cuda.Stream()

    states, packed = {}, {}
    for layer, variant in MATS:
        n, k = SHAPES[layer]
        st = mbp.prepare({layer: make_weight(n, k, variant, dev)})
        states[(layer, variant)] = st
        packed[(layer, variant)] = st["layers"][layer]
    torch.cuda.empty_cache()
    calls = []  # name, layer, variant, m, packed, x_dev, out_dev, x_host, out_host, bytes
    for m in MS:
        for layer, variant in MATS:
            n, k = SHAPES[layer]
            p = packed[(layer, variant)]
            x = make_x(m, k, dev)
            out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
            xh = x.cpu().pin_memory()
            oh = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
            nbytes = p.payload_bytes + p.bases.numel() + 2 * m * k + 2 * m * n
            calls.append((f"{layer}_m{m}_{variant}", layer, variant, m, p, x, out, xh, oh, nbytes))
    step_bytes = sum(c[-1] for c in calls)

    def step():
        for c in calls:
            mbp.gemv(c[4], c[5], out=c[6])

    g_step = graph_of(step, side)
    for _ in range(args.warmup):
        g_step.replay()
    torch.cuda.synchronize()
    assert mbp.device_status() == 0

    # ---------------- timed region: exactly K step replays ----------------
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a.record()
        for _ in range(args.steps):
            g_step.replay()
        b.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    clocks = clk.summary()
    step_ms = a.elapsed_time(b) / args.steps
    assert mbp.device_status() == 0, "device status word set during the timed region"
    if world > 1:
        t = torch.tensor([step_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms = float(t.item())
    value = step_bytes * world / (step_ms * 1e-3) / 1e12

    # ---------------- per-shape us/call: graph over rotating copies of one matrix ----------------
    shapes = {}
    reps = 24
    for (layer, variant), p0 in packed.items():
        nc = max(3, (400 << 20) // p0.units.numel())
        ps = [p0] + [mbp.PackedC12(p0.units.clone(), p0.bases, p0.esc_off, p0.esc, p0.n, p0.k, p0.n_esc)
                     for _ in range(nc - 1)]
        for c in calls:
            if (c[1], c[2]) != (layer, variant):
                continue
            g = graph_of(lambda: [mbp.gemv(ps[i % nc], c[5], out=c[6]) for i in range(reps)], side)
            g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (2 * reps)
            shapes[c[0]] = {"us": round(us, 2), "tbps": round(c[-1] / us / 1e6, 3), "bytes": c[-1]}
            del g
        del ps
        torch.cuda.empty_cache()

    # ---------------- e2e through the public API with host buffers ----------------
    # Each call: its x travels host -> device on a copy stream, kernel_fn runs on the compute stream as soon as
    # that copy lands, and its output travels device -> host on a second copy stream, so the 32 copies of a step
    # overlap the kernels of the other calls (a serving loop's usual double-buffering); the step ends when the
    # last output is on the host.
    h2d_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream()

    def api_step():
        comp = torch.cuda.current_stream()
        h2d_s.wait_stream(comp)
        d2h_s.wait_stream(comp)
        for c in calls:
            st = states[(c[1], c[2])]
            with torch.cuda.stream(h2d_s):
                xd = c[7].to(dev, non_blocking=True)
            comp.wait_stream(h2d_s)
            xd.record_stream(comp)
            out = mbp.kernel_fn({"x": xd, "config": {"m": c[3], "n": c[4].n, "k": c[4].k, "layer": c[1]}}, st)
            d2h_s.wait_stream(comp)
            with torch.cuda.stream(d2h_s):
                c[8].copy_(out, non_blocking=True)
            out.record_stream(d2h_s)
        comp.wait_stream(h2d_s)
        comp.wait_stream(d2h_s)

    for _ in range(max(1, args.warmup)):
        api_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, min(args.steps, 50))
    # eager: every call pays Python + launch overhead on the host (reported beside the headline)
    e0.record()
    for _ in range(e2e_steps):
        api_step()
    e1.record()
    torch.cuda.synchronize()
    eager_ms = e0.elapsed_time(e1) / e2e_steps
    # headline e2e: the same public-API step (pinned-host -> device copy of x, kernel_fn, device -> pinned-host
    # copy of the output, per call) captured once in a CUDA graph and replayed, as the reference's harness replays
    # kernel_fn
    g_api = graph_of(api_step, side)
    for _ in range(3):
        g_api.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(e2e_steps):
        g_api.replay()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    del g_api
    h2d = sum(2 * c[3] * c[4].k for c in calls)
    d2h = sum(2 * c[3] * c[4].n for c in calls)

    hbm, peak_kind = peaks()
    dom = [c[0] for c in calls if c[1] == "qkv_gate"]
    dom_bytes = sum(shapes[nm]["bytes"] for nm in dom)
    dom_us = sum(shapes[nm]["us"] for nm in dom)
    achieved = dom_bytes / (dom_us * 1e-6) / 1e9

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            v, dt, cores, sample = cpu_reference_run(1, 0, sample_rows=512)
            cpu = {"value": round(v, 6), "unit": "TB/s", "cores": cores, "kind": "port", "sample": sample}
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: W~N(0,0.02) torch seed 0 (+1% x256 variant, randperm seed 2), x~N(0,1) seed 1",
            "config": {"workload": "config2 decode GEMV: qkv_gate 6144->14336 and o 6144->6144, M in {1,8,16,32}, "
                                   "plain + 1% x256 escape weights (16 calls per step)",
                       "l2": "cold by construction: >=250 MB of other weights between reuses of a matrix "
                             "(inputs larger than L2), no flush kernel",
                       "timing": "CUDA-graph replay of the step, CUDA events on the replay stream",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": NCU_TRAFFIC_QKV_M1,
                         "kernel": "k_gemv, the 8 qkv_gate launches of a step", "peak_kind": f"{peak_kind} hbm_gbs",
                         "frac_of_8tbps": round(achieved / 8000.0, 4)},
            "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                    "timing": "CUDA-graph replay of the public-API step (per call: H2D of x on a copy stream, "
                              "kernel_fn, D2H of out on a second copy stream, overlapping the other calls)",
                    "eager_ms_per_step": round(eager_ms, 4)},
            "gpu_launches": len(calls) * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "shapes": shapes,
        }
        print(json.dumps(line), flush=True)


def run_mbp_tp(args, rank, world):
    """N > 1: the same 16-call step, each projection tensor-parallel over the N ranks (QKV+gate column-parallel
    + all-gather, O row-parallel + all-reduce of FP32 partials; by default through the GEMV's peer stores with
    the receive fused into it, `--transport nccl` for NCCL collectives).  Total work is fixed
    (strong scaling); value = packed bytes of the unsharded layers per step / step time (max over ranks)."""
    import torch
    import torch.distributed as dist
    import mbp
    from mbp.tp import TPLinear

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    lins = {}
    for layer, variant in MATS:
        n, k = SHAPES[layer]
        lins[(layer, variant)] = TPLinear(make_weight(n, k, variant, dev), "column" if layer == "qkv_gate" else "row",
                                          transport=args.transport)
    transport = next(iter(lins.values())).transport
    torch.cuda.empty_cache()
    shard_bytes = {key: torch.tensor([lin.payload_bytes], device=dev) for key, lin in lins.items()}
    for t in shard_bytes.values():
        dist.all_reduce(t)
    calls = []
    for m in MS:
        for layer, variant in MATS:
            n, k = SHAPES[layer]
            x = make_x(m, k, dev)
            nbytes = int(shard_bytes[(layer, variant)].item()) + 2 * m * k + 2 * m * n
            calls.append((f"{layer}_m{m}_{variant}", lins[(layer, variant)], x, nbytes, m, n, k))
    step_bytes = sum(c[3] for c in calls)

    def step():
        for c in calls:
            c[1](c[2])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    g = None
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                step()
        torch.cuda.synchronize()
        g = graph
    except Exception:
        g = None
    ok = torch.tensor([1 if g is not None else 0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    use_graph = int(ok.item()) == 1
    run = (lambda: g.replay()) if use_graph else step
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index) as clk:
        dist.barrier()
        torch.cuda.synchronize()
        a.record()
        for _ in range(args.steps):
            run()
        b.record()
        torch.cuda.synchronize()
        dist.barrier()
    clocks = clk.summary()
    t = torch.tensor([a.elapsed_time(b) / args.steps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    assert mbp.device_status() == 0

    # e2e: host x in, host output back, every call, through the layers' public forward: as at N = 1, each call's
    # x travels host -> device on a copy stream and its output device -> host on a second one, overlapping the
    # other calls, and the step is captured once in a CUDA graph and replayed (the eager time is reported beside)
    hx = [c[2].cpu().pin_memory() for c in calls]
    ho = [torch.empty((c[4], c[5]), dtype=torch.bfloat16).pin_memory() for c in calls]
    h2d_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream()

    def api_step():
        comp = torch.cuda.current_stream()
        h2d_s.wait_stream(comp)
        d2h_s.wait_stream(comp)
        for c, xh, oh in zip(calls, hx, ho):
            with torch.cuda.stream(h2d_s):
                xd = xh.to(dev, non_blocking=True)
            comp.wait_stream(h2d_s)
            xd.record_stream(comp)
            out = c[1](xd)
            d2h_s.wait_stream(comp)
            with torch.cuda.stream(d2h_s):
                oh.copy_(out, non_blocking=True)
            out.record_stream(d2h_s)
        comp.wait_stream(h2d_s)
        comp.wait_stream(d2h_s)

    def timed_max(run, n):
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            run()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / n], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    api_step()
    e2e_steps = max(3, min(args.steps, 20))
    eager_e2e_ms = timed_max(api_step, e2e_steps)
    g_api = None
    if use_graph:
        side2 = torch.cuda.Stream()
        side2.wait_stream(torch.cuda.current_stream())
        g_api = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side2):
            with torch.cuda.graph(g_api, stream=side2):
                api_step()
        torch.cuda.synchronize()
        for _ in range(3):
            g_api.replay()
    e2e_ms = timed_max(g_api.replay, e2e_steps) if g_api is not None else eager_e2e_ms
    hbm, peak_kind = peaks()
    if rank == 0:
        value = step_bytes / (step_ms * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: W~N(0,0.02) torch seed 0 (+1% x256 variant, randperm seed 2), x~N(0,1) seed 1",
            "config": {"workload": "config2 decode GEMV step (16 calls), tensor-parallel: qkv_gate column-parallel + "
                                   "all-gather, o row-parallel + all-reduce of FP32 partials",
                       "transport": ("one kernel per call: the shard GEMV stores epoch-tagged words into every "
                                     "rank's buffer over NVLink (CUDA IPC) and its CTAs assemble their tiles"
                                     if transport == "p2p" else "NCCL collectives"),
                       "l2": "cold by construction (>=250 MB of other weights between reuses of a matrix on one GPU "
                             "at N=1; per-GPU shards at N>1)",
                       "timing": ("CUDA-graph replay" if use_graph else "eager launches") +
                                 " of the step, CUDA events, max over ranks",
                       "parallelism": f"tp{world}"},
            "roofline": {"bound": "hbm", "achieved": round(value * 1e3 / world, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(value * 1e3 / world / hbm, 4), "traffic": None,
                         "kernel": "whole step per GPU (GEMV + collectives)", "peak_kind": f"{peak_kind} hbm_gbs"},
            "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
                    "h2d_bytes_per_step": sum(2 * c[4] * c[6] for c in calls),
                    "d2h_bytes_per_step": sum(2 * c[4] * c[5] for c in calls), "ms_per_step": round(e2e_ms, 4),
                    "timing": ("CUDA-graph replay" if g_api is not None else "eager launches") +
                              " of the public-API step (per call: H2D of x on a copy stream, the layer's forward, "
                              "D2H of out on a second copy stream, overlapping the other calls), max over ranks",
                    "eager_ms_per_step": round(eager_e2e_ms, 4)},
            # per call: the GEMV + the finish kernel (p2p) or the assemble / BF16-rounding kernel after NCCL
            "gpu_launches": 2 * len(calls) * args.steps,
            "clocks": clocks,
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    if g is not None:
        del g
    if g_api is not None:
        del g_api
    torch.cuda.synchronize()


# The reference's published per-shape times (us, NVIDIA H200, v18 submission, results/v18_shapes.csv:2-31) at its
# own layer shapes: (M, layer) -> us.  Weights: qkv_gate 2304x8192, o 8192x1024, pooler 4096x8192, unpooler
# 8192x4096 (n = 1024 at M <= 8), router FP32 256x8192.
REF_SHAPES = {"qkv_gate": (2304, 8192), "o": (8192, 1024), "pooler": (4096, 8192), "unpooler": (8192, 4096),
              "router": (256, 8192)}
REF_H200_US = {
    (1, "qkv_gate"): 9.34, (1, "o"): 5.10, (1, "pooler"): 13.29, (1, "unpooler"): 3.72, (1, "router"): 3.94,
    (8, "qkv_gate"): 9.69, (8, "o"): 5.50, (8, "pooler"): 13.61, (8, "unpooler"): 4.28, (8, "router"): 4.34,
    (16, "qkv_gate"): 10.25, (16, "o"): 5.48, (16, "pooler"): 13.98, (16, "unpooler"): 13.74, (16, "router"): 4.23,
    (32, "qkv_gate"): 12.16, (32, "o"): 5.81, (32, "pooler"): 16.13, (32, "unpooler"): 15.60, (32, "router"): 5.04,
    (128, "qkv_gate"): 13.99, (128, "o"): 6.89, (128, "pooler"): 20.49, (128, "unpooler"): 19.37,
    (128, "router"): 6.19,
    (256, "qkv_gate"): 17.09, (256, "o"): 8.98, (256, "pooler"): 24.19, (256, "unpooler"): 23.32,
    (256, "router"): 8.44,
}


def run_ref_shapes(reps: int = 200):
    """--ref-shapes: kernel_fn at the reference's 30 (M, layer) shapes with cold L2, as its judge timed them (CUDA
    graph of one call with a new output tensor, L2 flushed between calls, fixed replay overhead excluded).  CUDA
    events on this box resolve 2.048 us, too coarse around a single replay, so each shape is timed by difference:
    `reps` calls as replays of a graph of 10 x [flush a 256 MB buffer, call] minus the flushes alone, each between
    one pair of events, divided by `reps`.  One JSON line; the H200 numbers are the reference's, on different
    hardware (4.8 vs 8 TB/s HBM)."""
    import torch
    import mbp
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    ws = {name: (torch.randn(n, k) * 0.02).to(torch.bfloat16).to(dev)
          for name, (n, k) in REF_SHAPES.items() if name != "router"}
    ws["router"] = (torch.randn(256, 8192) * 0.01).to(dev)
    mbp.prepare({"o": ws["o"]})  # library load and first-call setup, outside the prepare timings
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    st = mbp.prepare(ws)  # GPU packing + device round-trip verification of all five layers
    torch.cuda.synchronize()
    prep = {"prepare_s": round(time.perf_counter() - t0, 3)}
    with tempfile.TemporaryDirectory() as td:
        cache = os.path.join(td, "weights.mbp")
        t0 = time.perf_counter()
        mbp.prepare(ws, cache=cache)
        torch.cuda.synchronize()
        prep["prepare_and_write_cache_s"] = round(time.perf_counter() - t0, 3)
        t0 = time.perf_counter()
        mbp.prepare(ws, cache=cache)
        torch.cuda.synchronize()
        prep["prepare_from_cache_s"] = round(time.perf_counter() - t0, 3)
        prep["cache_bytes"] = os.path.getsize(cache)
    prep["reference_h200_prepare_s"] = 53.80  # cold prepare of the reference, results/v18.json:15
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    inner = 10  # pairs per graph: a graph replay's duration comes in whole 2.048 us ticks on this box

    def graph_time(fn):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(inner):
                fn()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps // inner):
            g.replay()
        b.record()
        b.synchronize()
        del g
        return a.elapsed_time(b) * 1e3 / (reps // inner * inner)

    # Copies of each layer's packed weights (same descriptors, cloned payload) so that back-to-back calls rotate
    # over more than 2x L2 of weights: every call reads its weights from HBM, as in a decode loop.
    from mbp.ops import PackedC12, PackedHiLo

    def copies_of(layer):
        if layer in st["hilo"]:
            p = st["hilo"][layer]
            reps_ = max(2, -(-(256 << 20) // p.units.numel()))
            ps = [p] + [PackedHiLo(p.units.clone(), p.n, p.k) for _ in range(reps_ - 1)]
            return [{"layers": {}, "hilo": {layer: q}, "k": st["k"]} for q in ps]
        p = st["layers"][layer]
        reps_ = max(2, -(-(256 << 20) // p.units.numel()))
        ps = [p] + [PackedC12(p.units.clone(), p.bases, p.esc_off, p.esc, p.n, p.k, p.n_esc) for _ in range(reps_ - 1)]
        return [{"layers": {layer: q}, "hilo": {}, "k": st["k"]} for q in ps]

    rows, ratios = [], []
    for layer in REF_SHAPES:
        states = copies_of(layer)
        for (m, lay), ref_us in REF_H200_US.items():
            if lay != layer:
                continue
            n, k = REF_SHAPES[layer]
            n_call = 1024 if layer == "unpooler" and m <= 8 else n
            x = make_x(m, k, dev)
            data = {"x": x, "config": {"m": m, "n": n_call, "k": k, "layer": layer}}

            def rotate():
                for s in states:
                    mbp.kernel_fn(data, s)

            def flush_call():
                torch.amax(flush)  # read flush: L2 left holding clean lines
                mbp.kernel_fn(data, st)

            row = {"m": m, "layer": layer, "n": n_call, "k": k,
                   "us": round(graph_time(rotate) / len(states), 2),
                   "us_after_flush": round(graph_time(flush_call) - graph_time(lambda: torch.amax(flush)), 2),
                   "ref_h200_us": ref_us}
            row["ratio_ref_over_this"] = round(ref_us / row["us"], 3)
            rows.append(row)
            ratios.append(ref_us / row["us"])
        del states
    assert mbp.device_status() == 0
    import math
    geo = math.exp(sum(math.log(r) for r in ratios) / len(ratios))
    print(json.dumps({"ref_shapes": sorted(rows, key=lambda r: (r["m"], list(REF_SHAPES).index(r["layer"]))),
                      "geomean_ratio_vs_ref_h200": round(geo, 3), "prepare": prep,
                      "method": "us: back-to-back kernel_fn calls in CUDA-graph replays, rotating over copies of the "
                                "layer's packed weights totalling >= 256 MB (every call reads cold weights), %d "
                                "calls per copy-cycle group, one event pair; us_after_flush: (10 x [read 256 MB, call]"
                                " - the reads alone) per call, which adds the kernel-boundary transition after a "
                                "foreign kernel" % reps}),
          flush=True)


def run_profile(spec: str, launches: int = 3):
    """--profile LAYER:M:VARIANT -- a few launches of one call for an ncu capture (no timing, no output)."""
    import torch
    import mbp
    layer, m, variant = spec.split(":")
    n, k = SHAPES[layer]
    torch.cuda.set_device(0)
    st = mbp.prepare({layer: make_weight(n, k, variant, "cuda")})
    x = make_x(int(m), k, "cuda")
    for _ in range(launches):
        mbp.kernel_fn({"x": x, "config": {"m": int(m), "n": n, "k": k, "layer": layer}}, st)
    torch.cuda.synchronize()
    assert mbp.device_status() == 0
    path = st["layers"][layer].plan(int(m)).as_tuple() if int(m) <= mbp.GEMV_MAX_M else "tcgen05 gemm"
    print("profile run ok:", spec, path)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile", default=None, help="LAYER:M:VARIANT: a few launches of one call, for ncu")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mbp", choices=["mbp", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--ref-shapes", action="store_true",
                    help="time kernel_fn at the reference's 30 published shapes (one JSON line, not the bench line)")
    ap.add_argument("--transport", default="auto", choices=["auto", "p2p", "nccl"],
                    help="N > 1: tensor-parallel exchange (auto = GEMV peer stores on one node)")
    args = ap.parse_args()
    if args.profile:
        run_profile(args.profile)
        return
    if args.ref_shapes:
        run_ref_shapes()
        return
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        if args.impl == "mbp":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif world > 1:
            run_mbp_tp(args, rank, world)
        else:
            run_mbp(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
