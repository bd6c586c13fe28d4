"""Benchmark of the small-M projection on B200 (BASELINE.json config 2 at N=1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mbp|reference]

One STEP = one cold-L2 call of each decode-GEMV shape of BASELINE config 2: fused QKV+gate (K=6144, N=14336) and
O (K=N=6144) at M in {1, 8, 16, 32}, each with plain N(0, 0.02) weights and with the 1%-x256 escape variant
(16 calls).  Before every call a 512 MB buffer is written to flush L2 (outside the timed events); each call is
timed with CUDA events on the launching stream.  value = packed weight bytes streamed / kernel time (TB/s),
the BASELINE metric's bandwidth form; per-shape us/call are in "shapes".

--impl reference runs the reference path's CPU implementation (the C port of the oracle: decode + FP32
accumulate, all host threads) on a bounded row sample of the same workload, rank 0 only.
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
VARIANTS = ("plain", "esc1pct")
FLUSH_BYTES = 512 << 20


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
    """Samples nvidia-smi clocks / throttle reasons while the timed region runs."""

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
                                       "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
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
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_run(steps: int, warmup: int, sample_rows: int = 256):
    """The reference path on the host: the oracle's C port (decode + FP32 accumulate) over all host threads on a
    bounded row sample of every shape.  Returns (TB/s of packed weights, seconds per sampled step, cores)."""
    import numpy as np
    import torch
    from oracle import oracle
    cores = os.cpu_count() or 1
    work = []
    for layer, (n, k) in SHAPES.items():
        for variant in VARIANTS:
            w = make_weight(sample_rows, k, variant, "cpu")
            p = oracle.pack(w.view(torch.int16).numpy().view(np.uint16), tile_base=True)
            for m in MS:
                x = make_x(m, k, "cpu").view(torch.int16).numpy().view(np.uint16)
                work.append((p, x, sample_rows * k * 1.5 + p["esc"].size * 4))
    for _ in range(warmup):
        for p, x, _b in work:
            oracle.gemv_packed(x, p, threads=cores)
    t0 = time.perf_counter()
    for _ in range(steps):
        for p, x, _b in work:
            oracle.gemv_packed(x, p, threads=cores)
    dt = (time.perf_counter() - t0) / max(steps, 1)
    nbytes = sum(b for _, _, b in work)
    return nbytes / dt / 1e12, dt, cores, f"{sample_rows} rows of each of the {len(work)} (layer, M, variant) calls"


def run_reference(args, rank, world):
    if rank != 0:
        return
    steps = max(1, min(args.steps, 3))
    warm = min(args.warmup, 1)
    v, dt, cores, sample = cpu_reference_run(steps, warm)
    line = {"metric": METRIC, "value": round(v, 6), "unit": "TB/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warm, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (BASELINE.json config 2 recipe)",
            "config": {"workload": "config2 decode GEMV: qkv_gate 6144->14336, o 6144->6144, M in {1,8,16,32}, "
                                   "plain + 1% x256 escape variant", "l2": "n/a (host)"},
            "impl": "reference",
            "cpu_baseline": {"value": round(v, 6), "unit": "TB/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 6), "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_mbp(args, rank, world):
    import torch
    import torch.distributed as dist
    import mbp

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    calls = []  # (name, layer, variant, m, packed, x_dev, x_host, out_host, bytes)
    states = {}
    for layer, (n, k) in SHAPES.items():
        for variant in VARIANTS:
            w = make_weight(n, k, variant, dev)
            st = mbp.prepare({layer: w})
            states[(layer, variant)] = st
            p = st["layers"][layer]
            del w
            for m in MS:
                x = make_x(m, k, dev)
                xh = x.cpu().pin_memory()
                oh = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
                nbytes = p.payload_bytes + 2 * m * k + 2 * m * n + p.bases.numel()
                calls.append((f"{layer}_m{m}_{variant}", layer, variant, m, p, x, xh, oh, nbytes))
    torch.cuda.synchronize()

    def one_step(times=None, e2e=None):
        for i, (name, layer, variant, m, p, x, xh, oh, nbytes) in enumerate(calls):
            flush.fill_(float(i))
            st = states[(layer, variant)]
            if e2e is None:
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                mbp.gemv(p, x)
                b.record(stream)
                if times is not None:
                    times[i].append((a, b))
            else:
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                xd = xh.to(dev, non_blocking=True)
                out = mbp.kernel_fn({"x": xd, "config": {"m": m, "n": p.n, "k": p.k, "layer": layer}}, st)
                oh.copy_(out, non_blocking=True)
                b.record(stream)
                e2e[i].append((a, b))

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    times = [[] for _ in calls]
    with Clocks(dev.index) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            one_step(times)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        if world > 1:
            dist.barrier()
    clocks = clk.summary()
    assert mbp.device_status() == 0, "device status word set during the timed region"

    per_call_ms = [[a.elapsed_time(b) for a, b in ts] for ts in times]
    step_ms = sum(statistics.mean(v) for v in per_call_ms)
    total_bytes = sum(c[-1] for c in calls)
    if world > 1:
        t = torch.tensor([step_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms = float(t.item())
    value = total_bytes * world / (step_ms * 1e-3) / 1e12

    # end-to-end through the public API with host buffers (H2D of x and D2H of out inside the timed region)
    e2e = [[] for _ in calls]
    for _ in range(max(1, args.warmup // 2)):
        one_step(e2e=[[] for _ in calls])
    torch.cuda.synchronize()
    for _ in range(args.steps):
        one_step(e2e=e2e)
    torch.cuda.synchronize()
    e2e_ms = sum(statistics.mean(a.elapsed_time(b) for a, b in ts) for ts in e2e)
    h2d = sum(2 * c[3] * c[4].k for c in calls)
    d2h = sum(2 * c[3] * c[4].n for c in calls)

    # roofline of the dominant kernel: the QKV+gate GEMV launches
    hbm, peak_kind = peaks()
    dom = [i for i, c in enumerate(calls) if c[1] == "qkv_gate"]
    dom_bytes = sum(calls[i][-1] for i in dom)
    dom_ms = sum(statistics.mean(per_call_ms[i]) for i in dom)
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    shapes = {c[0]: {"us": round(statistics.median(per_call_ms[i]) * 1e3, 2),
                     "tbps": round(c[-1] / (statistics.median(per_call_ms[i]) * 1e-3) / 1e12, 3)}
              for i, c in enumerate(calls)}

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            v, dt, cores, sample = cpu_reference_run(1, 0, sample_rows=128)
            cpu = {"value": round(v, 6), "unit": "TB/s", "cores": cores, "kind": "port", "sample": sample}
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: W~N(0,0.02) torch seed 0 (+1% x256 variant, randperm seed 2), x~N(0,1) seed 1",
            "config": {"workload": "config2 decode GEMV: qkv_gate 6144->14336, o 6144->6144, M in {1,8,16,32}, "
                                   "plain + 1% x256 escape variant (16 calls per step)",
                       "l2": "flushed before every call (512 MB write, outside the timed events)",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": None,
                         "kernel": "k_gemv (qkv_gate launches)", "peak_kind": peak_kind,
                         "frac_of_8tbps": round(achieved / 8000.0, 4)},
            "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": len(calls) * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "shapes": shapes,
            "wall_s_timed": round(wall, 3),
        }
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mbp", choices=["mbp", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    args = ap.parse_args()
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
        else:
            run_mbp(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
