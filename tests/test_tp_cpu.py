"""Tensor-parallel host logic on CPU ranks (gloo, world size 2): the sharding plan, the collective choreography
and the output assembly reproduce the unsharded projection; a rank that disappears makes the survivor's
collective fail within the process-group timeout instead of hanging; the peer-store transport is chosen only for
ranks on GPUs of their own.  The local products are computed by the CPU oracle (each rank packs its own shard with
its own exponent bases and escapes), so no GPU is involved."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_DIR, ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _setup(rank, world, port, timeout_s=60):
    import sys
    for p in (ROOT, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_parity(rank, world, port, errq):
    try:
        _setup(rank, world, port)
        from mbp.tp import TPPlan
        from oracle import oracle
        g = torch.Generator().manual_seed(0)
        n, k = 256, 512
        w = (torch.randn(n, k, generator=g) * 0.02)
        idx = torch.randperm(n * k, generator=torch.Generator().manual_seed(2))[: n * k // 100]
        w.view(-1)[idx] *= 256
        w = w.to(torch.bfloat16)
        for m in (1, 5, 32):
            x = torch.randn(m, k, generator=g).to(torch.bfloat16)
            full = torch.from_numpy(oracle.linear_f64(_bits(x), _bits(w))).float()
            # column-parallel: shard rows, gather rank-major, assemble [m, n]
            plan = TPPlan("column", world, rank, n, k)
            pk = oracle.pack(_bits(plan.shard(w)), tile_base=True)
            local, _ = oracle.gemv_packed(_bits(plan.x_slice(x)), pk)
            parts = [torch.empty_like(torch.from_numpy(local)) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(local))
            gathered = torch.stack(parts)                               # [P, m, n/P]
            out = gathered.permute(1, 0, 2).reshape(m, n)
            assert torch.allclose(out, full, rtol=1e-4, atol=1e-4), ("column", m)
            # row-parallel: shard columns, FP32 partials, all-reduce; reduce-scatter keeps a column slice
            plan = TPPlan("row", world, rank, n, k)
            pk = oracle.pack(_bits(plan.shard(w)), tile_base=True)
            part, _ = oracle.gemv_packed(_bits(plan.x_slice(x)), pk)
            part = torch.from_numpy(part)
            red = part.clone()
            dist.all_reduce(red)
            assert torch.allclose(red, full, rtol=1e-4, atol=1e-4), ("row", m)
            c0, c1 = plan.scatter_cols()
            assert torch.allclose(red[:, c0:c1], full[:, rank * n // world:(rank + 1) * n // world], rtol=1e-4,
                                  atol=1e-4), ("scatter", m)
            # every rank's shard round-trips through the per-shard packing exactly
            assert np.array_equal(oracle.unpack(pk), _bits(plan.shard(w)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_tp_plan_parity_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    procs = [ctx.Process(target=_worker_parity, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert all(p.exitcode == 0 for p in procs), errs


def _worker_missing(rank, world, port, q):
    _setup(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(3)  # leaves between steps, with no collective in flight
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put("rank0-no-error")
    except Exception as e:
        q.put(f"rank0-error:{type(e).__name__}")


def test_tp_missing_rank_times_out():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_missing, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    msgs = []
    while not q.empty():
        msgs.append(q.get())
    assert procs[1].exitcode == 3
    assert any(m.startswith("rank0-error") for m in msgs), msgs
    for p in procs:
        if p.is_alive():
            p.kill()


def test_plan_rules():
    from mbp.tp import TPPlan
    p = TPPlan("column", 4, 2, 14336, 6144)
    assert p.rows == (7168, 10752) and p.cols == (0, 6144)
    q = TPPlan("row", 8, 7, 6144, 6144)
    assert q.cols == (5376, 6144) and q.rows == (0, 6144) and q.scatter_cols() == (5376, 6144)
    with pytest.raises(ValueError):
        TPPlan("row", 8, 0, 6144, 6000)
    with pytest.raises(ValueError):
        TPPlan("column", 3, 0, 6144 + 16, 6144)


def test_peer_store_placement_rule():
    """The peer-store transport (kernels that wait on each other's stores) is chosen only when every rank has a
    GPU of its own on this host, at most 8 ranks, and every visible peer is peer-accessible; anything else falls
    back to NCCL."""
    from mbp.tp import _p2p_placement_ok
    local = {f"GPU-{i}": i for i in range(8)}

    def peers(a, b):
        return True

    def seen(uuids, hosts=None):
        return [((hosts or {}).get(i, "h"), u) for i, u in enumerate(uuids)]

    assert _p2p_placement_ok(seen(["GPU-0", "GPU-1"]), "h", local, 0, peers)
    assert _p2p_placement_ok(seen([f"GPU-{i}" for i in range(8)]), "h", local, 3, peers)
    assert not _p2p_placement_ok(seen(["GPU-0", "GPU-0"]), "h", local, 0, peers)          # two ranks, one GPU
    assert not _p2p_placement_ok(seen(["GPU-0", "GPU-1"], {1: "other"}), "h", local, 0, peers)  # two hosts
    assert not _p2p_placement_ok(seen([f"GPU-{i}" for i in range(9)]), "h", dict(local, **{"GPU-8": 8}), 0, peers)
    assert not _p2p_placement_ok(seen(["GPU-0", "GPU-1"]), "h", local, 0, lambda a, b: False)  # no peer access
    # a peer this process cannot see (per-rank device lists): its buffer's IPC mapping is unknown, so NCCL
    assert not _p2p_placement_ok(seen(["GPU-0", "GPU-5"]), "h", {"GPU-0": 0}, 0, peers)


def test_row_exchange_choice():
    from mbp.tp import row_exchange_for
    assert row_exchange_for(2) == "sum" and row_exchange_for(4) == "rsag" and row_exchange_for(8) == "rsag"
    assert row_exchange_for(8, "sum") == "sum" and row_exchange_for(2, "rsag") == "rsag"
    with pytest.raises(ValueError):
        row_exchange_for(4, "ring")


def test_exchange_route():
    """Which exchange each call takes (the GPU paths themselves are checked by tests/tp_worker.py)."""
    from mbp.tp import exchange_route as r
    assert r("column", "all", 4, 1, True) == "gemv-p2p" and r("row", "all", 8, 32, True) == "gemv-p2p"
    assert r("row", "scatter", 2, 8, True) == "nccl"
    assert r("column", "all", 8, 33, True) == "gemm-p2p" and r("column", "all", 8, 256, True) == "gemm-p2p"
    assert r("column", "all", 8, 257, True) == "nccl"
    assert r("row", "all", 2, 256, True) == "gemm-p2p" and r("row", "all", 4, 256, True) == "nccl"
    assert r("column", "all", 2, 8, False) == "nccl"


def _worker_forward(rank, world, port, errq):
    """TPLinear.forward's collective path on gloo ranks: routing, the collectives and the shapes around them, with
    the device kernels (shard GEMV/GEMM, assembly, BF16 rounding) replaced by CPU equivalents of the oracle."""
    try:
        _setup(rank, world, port)
        from types import SimpleNamespace
        from mbp.tp import TPLinear, TPPlan
        from oracle import oracle
        g = torch.Generator().manual_seed(0)
        n, k = 128, 256
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        for mode, reduce in (("column", "all"), ("row", "all")):
            lin = object.__new__(TPLinear)
            lin.plan = TPPlan(mode, world, rank, n, k)
            lin.reduce, lin.group, lin._xbuf = reduce, None, None
            lin.packed = SimpleNamespace(units=torch.empty(0))
            pk = oracle.pack(_bits(lin.plan.shard(w)), tile_base=True)

            def local(x, dt, pk=pk, lin=lin):
                out, _ = oracle.gemv_packed(_bits(lin.plan.x_slice(x)), pk)
                return torch.from_numpy(out).to(dt)

            lin._local = local
            lin._assemble = lambda gathered, m, ns, lin=lin: (
                gathered.view(world, m, ns).permute(1, 0, 2).reshape(m, lin.plan.n))
            lin._to_bf16 = lambda part: part.to(torch.bfloat16)
            for m in (1, 40, 300):  # the GEMV, GEMM and beyond-exchange sizes all take the collective path here
                x = torch.randn(m, k, generator=g).to(torch.bfloat16)
                full = torch.from_numpy(oracle.linear_f64(_bits(x), _bits(w))).float()
                out = lin.forward(x)
                assert out.shape == (m, n) and out.dtype == torch.bfloat16, (mode, m, out.shape)
                assert torch.allclose(out.float(), full, rtol=1e-2, atol=1e-2), (mode, m)
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_tp_forward_collective_path_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    procs = [ctx.Process(target=_worker_forward, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert all(p.exitcode == 0 for p in procs), errs
