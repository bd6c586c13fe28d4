"""Worker of tests/test_gpu_tp.py: one rank of a tensor-parallel check (launched by torchrun).

Column-parallel fused QKV+gate (K=6144, N=14336, all-gather) and row-parallel output
projection (K=N=6144, all-reduce and reduce-scatter) at M in {1, 8, 32, 256}, through every transport (NCCL
collectives; the GEMV's epoch-tagged peer stores with the receive fused into the GEMV -- row-parallel as an
all-to-all of the partials or as a reduce-scatter to each tile's owner plus a gather -- and with the separate
receive kernel), checked against the FP32 reference of the unsharded projection (rtol 1e-2 / atol 1e-2).  The
peer-store paths are also checked for: identical bits on every rank, identical column outputs to the NCCL path
(same per-shard GEMV), identical row outputs of the fused and two-kernel forms, back-to-back calls alternating
the exchange buffers, and replay of a captured CUDA graph.  Then the collective teardown (the exchange buffers'
memory returns, released layers refuse calls) and the drop-in pair prepare_tp / kernel_fn_tp.  Exits non-zero on
any mismatch."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "muse-bf16-proj_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

RTOL = ATOL = 1e-2


def _bad(out, ref):
    err = (out.float() - ref).abs()
    return int((err > ATOL + RTOL * ref.abs()).sum()) + int((~torch.isfinite(out.float())).sum()), float(err.max())


def _same_on_all_ranks(t: torch.Tensor) -> bool:
    world = dist.get_world_size()
    got = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(got, t.contiguous())
    return all(torch.equal(got[0], g) for g in got)


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    import mbp
    from mbp.tp import TPLinear, kernel_fn_tp, prepare_tp, release_tp
    fails = []

    def fail(msg):
        fails.append(msg)
        print(f"rank {rank} {msg}", flush=True)

    g = torch.Generator().manual_seed(0)
    w_qkv = (torch.randn(14336, 6144, generator=g) * 0.02).to(torch.bfloat16).cuda()
    w_o = (torch.randn(6144, 6144, generator=g) * 0.02)
    idx = torch.randperm(w_o.numel(), generator=torch.Generator().manual_seed(2))[: w_o.numel() // 100]
    w_o.view(-1)[idx] *= 256
    w_o = w_o.to(torch.bfloat16).cuda()
    layers = {}
    for tr in ("nccl", "p2p", "p2p-two-kernels"):
        kw = {"transport": "p2p", "fused": False} if tr == "p2p-two-kernels" else {"transport": tr}
        layers[tr] = {"column": TPLinear(w_qkv, "column", **kw),
                      "row-all": TPLinear(w_o, "row", reduce="all", **kw)}
    layers["nccl"]["row-scatter"] = TPLinear(w_o, "row", reduce="scatter", transport="nccl")
    # both fused row-parallel exchanges at every P (the default picks the reduce-scatter + gather from 4 ranks on)
    layers["p2p-rsag"] = {"row-all": TPLinear(w_o, "row", reduce="all", transport="p2p", row_exchange="rsag")}
    layers["p2p-sum"] = {"row-all": TPLinear(w_o, "row", reduce="all", transport="p2p", row_exchange="sum")}
    if layers["p2p"]["column"].transport != "p2p":
        fail("p2p transport not selected")
    weights = {"column": w_qkv, "row-all": w_o, "row-scatter": w_o}

    # 1. every layer, every m, against the FP32 reference
    for m in (1, 8, 32, 100, 256):
        x = torch.randn(m, 6144, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16).cuda()
        for tr, ls in layers.items():
            for name, lin in ls.items():
                out = lin(x).clone()
                ref = x.float() @ weights[name].float().T
                if name == "row-scatter":
                    c0, c1 = lin.plan.scatter_cols()
                    ref = ref[:, c0:c1]
                bad, mx = _bad(out, ref)
                if bad:
                    fail(f"{tr} {name} m={m}: {bad} elements outside tolerance, max err {mx}")
                if tr.startswith("p2p") and not _same_on_all_ranks(out):
                    fail(f"{tr} {name} m={m}: ranks disagree")
                if tr.startswith("p2p") and name == "column":
                    if not torch.equal(out, layers["nccl"]["column"](x)):
                        fail(f"{tr} column m={m}: differs from the NCCL path")
                if tr == "p2p-two-kernels" and m <= 32 and name == "row-all":
                    for other in ("p2p", "p2p-rsag", "p2p-sum"):
                        if not torch.equal(out, layers[other]["row-all"](x)):
                            fail(f"row m={m}: the {other} and the two-kernel exchange differ")

    # 2. back-to-back calls on one stream (the exchange buffers alternate); outputs read before the next call
    col, row = layers["p2p"]["column"], layers["p2p"]["row-all"]
    xs = [torch.randn(8, 6144, generator=torch.Generator().manual_seed(100 + i)).to(torch.bfloat16).cuda()
          for i in range(6)]
    kept = []
    for x in xs:
        a = col(x)
        kept.append(a.clone())
        kept.append(row(a[:, :6144].contiguous()).clone())
    for i, x in enumerate(xs):
        ref_a = x.float() @ w_qkv.float().T
        bad, mx = _bad(kept[2 * i], ref_a)
        if bad:
            fail(f"p2p back-to-back column call {i}: {bad} bad, max err {mx}")
        ref_b = kept[2 * i][:, :6144].float() @ w_o.float().T
        bad, mx = _bad(kept[2 * i + 1], ref_b)
        if bad:
            fail(f"p2p back-to-back row call {i}: {bad} bad, max err {mx}")

    # 3. a captured CUDA graph of column -> row, replayed with new inputs
    xin = torch.zeros(4, 6144, dtype=torch.bfloat16, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            yb = row(col(xin)[:, :6144].contiguous())
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ya = col(xin)
        yb = row(ya[:, :6144].contiguous())
        yc = yb.clone()
    for i in range(4):
        xin.copy_(torch.randn(4, 6144, generator=torch.Generator().manual_seed(200 + i)).to(torch.bfloat16))
        graph.replay()
        ref_a = xin.float() @ w_qkv.float().T
        bad, mx = _bad(ya, ref_a)
        if bad:
            fail(f"p2p graph replay {i} (column): {bad} bad, max err {mx}")
        ref_b = ya[:, :6144].float() @ w_o.float().T   # from the projection's own BF16 intermediate
        bad, mx = _bad(yc, ref_b)
        if bad:
            fail(f"p2p graph replay {i} (row): {bad} bad, max err {mx}")
    del graph

    torch.cuda.synchronize()
    if mbp.device_status() != 0:
        fail("device status set")

    # 4. collective teardown: the exchange buffers (cudaMalloc'd outside torch's cache) go back to the device and
    # a released layer refuses further calls
    xbytes = sum(lin._xbuf.nbytes for ls in layers.values() for lin in ls.values() if lin._xbuf is not None)
    free0 = torch.cuda.mem_get_info()[0]
    for tr in ("nccl", "p2p", "p2p-two-kernels", "p2p-rsag", "p2p-sum"):
        release_tp({"tp": layers[tr]})
    torch.cuda.synchronize()
    freed = torch.cuda.mem_get_info()[0] - free0
    if freed < xbytes // 2:
        fail(f"teardown freed {freed} bytes of {xbytes} exchange bytes")
    try:
        col(xs[0])
        fail("a released layer accepted a call")
    except RuntimeError:
        pass

    # 5. the drop-in pair prepare_tp / kernel_fn_tp (QKV+gate column-parallel, O row-parallel), then its release
    st = prepare_tp({"qkv_gate": w_qkv, "o": w_o})
    x8 = xs[0]
    a = kernel_fn_tp({"x": x8, "config": {"m": 8, "n": 14336, "k": 6144, "layer": "qkv_gate"}}, st).clone()
    a6 = a[:, :6144].contiguous()
    b = kernel_fn_tp({"x": a6, "config": {"m": 8, "n": 6144, "k": 6144, "layer": "o"}}, st).clone()
    for name, out, ref in (("qkv_gate", a, x8.float() @ w_qkv.float().T), ("o", b, a6.float() @ w_o.float().T)):
        bad, mx = _bad(out, ref)
        if bad:
            fail(f"kernel_fn_tp {name}: {bad} bad, max err {mx}")
        if not _same_on_all_ranks(out):
            fail(f"kernel_fn_tp {name}: ranks disagree")
    release_tp(st)
    flag = torch.tensor([1 if fails else 0], device="cuda")
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if rank == 0:
        print("TP check", "ok" if int(flag.item()) == 0 else "FAILED", flush=True)
    sys.exit(0 if int(flag.item()) == 0 else 1)


if __name__ == "__main__":
    main()
