"""Worker of tests/test_gpu_tp.py: one rank of a tensor-parallel check over NCCL (launched by torchrun).

column-parallel fused QKV+gate (K=6144, N=14336, all-gather) and row-parallel output
projection (K=N=6144, all-reduce and reduce-scatter) at M in {1, 32, 256}, checked against the FP32 reference of
the unsharded projection (rtol 1e-2 / atol 1e-2).  Exits non-zero on any mismatch."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "muse-bf16-proj_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    import mbp
    from mbp.tp import TPLinear
    ok = True
    g = torch.Generator().manual_seed(0)
    w_qkv = (torch.randn(14336, 6144, generator=g) * 0.02).to(torch.bfloat16).cuda()
    w_o = (torch.randn(6144, 6144, generator=g) * 0.02)
    idx = torch.randperm(w_o.numel(), generator=torch.Generator().manual_seed(2))[: w_o.numel() // 100]
    w_o.view(-1)[idx] *= 256
    w_o = w_o.to(torch.bfloat16).cuda()
    col = TPLinear(w_qkv, "column")
    row_all = TPLinear(w_o, "row", reduce="all")
    row_sc = TPLinear(w_o, "row", reduce="scatter")
    for m in (1, 32, 256):
        x = torch.randn(m, 6144, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16).cuda()
        for name, lin, w, cols in (("column", col, w_qkv, None), ("row-all", row_all, w_o, None),
                                   ("row-scatter", row_sc, w_o, row_sc.plan.scatter_cols())):
            out = lin(x)
            ref = x.float() @ w.float().T
            if cols is not None:
                ref = ref[:, cols[0]:cols[1]]
            err = (out.float() - ref).abs()
            bad = int((err > 1e-2 + 1e-2 * ref.abs()).sum())
            if bad or not bool(torch.isfinite(out).all()):
                ok = False
                print(f"rank {rank} {name} m={m}: {bad} elements outside tolerance, max err {float(err.max())}",
                      flush=True)
    torch.cuda.synchronize()
    if mbp.device_status() != 0:
        ok = False
        print(f"rank {rank}: device status set", flush=True)
    flag = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if rank == 0:
        print("TP check", "ok" if int(flag.item()) == 0 else "FAILED", flush=True)
    sys.exit(0 if int(flag.item()) == 0 else 1)


if __name__ == "__main__":
    main()
