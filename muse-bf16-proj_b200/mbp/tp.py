"""Tensor-parallel projections over NCCL (torch.distributed), one process per GPU.

The reference is single-GPU; this layer shards its projections across P GPUs of one node:

* **column-parallel** (the fused QKV+gate projection): rank r packs rows [r*N/P, (r+1)*N/P) of W, computes its
  [m, N/P] shard with the GEMV (m <= 32) or the tcgen05 GEMM, and one NCCL all-gather of the BF16 shards plus
  ``mbp_tp_assemble_columns`` yields the full [m, N] output on every rank;
* **row-parallel** (the output projection): rank r packs columns [r*K/P, (r+1)*K/P), computes FP32 partial sums
  of the full [m, N] output from its slice of x, and an NCCL all-reduce (``reduce="all"``, full output on every
  rank) or reduce-scatter (``reduce="scatter"``, rank r keeps columns [r*N/P, (r+1)*N/P)) sums them before the
  BF16 rounding (``mbp_f32_to_bf16``).  Keeping the partials in FP32 preserves the single-GPU "FP32-accumulated"
  semantics up to summation order.

Each rank packs its own shard (per-shard exponent bases and escape lists).  Every rank must issue the same
collectives in the same order; all of them run on the current CUDA stream, so a step can be captured in a CUDA
graph.  ``TPPlan`` holds the host-side sharding and assembly rules on their own (tested with gloo CPU ranks).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ._lib import check, lib
from .ops import BASE_TILE, PackedC12, gemm, gemv, pack_c12

GEMV_MAX_M = 32


@dataclass(frozen=True)
class TPPlan:
    """Sharding of one projection W[n, k] over `world` ranks."""
    mode: str    # "column" (split n) or "row" (split k)
    world: int
    rank: int
    n: int
    k: int

    def __post_init__(self):
        if self.mode not in ("column", "row"):
            raise ValueError(self.mode)
        if self.mode == "column" and self.n % (16 * self.world):
            raise ValueError(f"column-parallel needs n % (16*P) == 0, n={self.n}, P={self.world}")
        if self.mode == "row" and self.k % (64 * self.world):
            raise ValueError(f"row-parallel needs k % (64*P) == 0, k={self.k}, P={self.world}")

    @property
    def rows(self) -> tuple[int, int]:
        """Weight rows (output columns) this rank owns."""
        if self.mode == "row":
            return 0, self.n
        s = self.n // self.world
        return self.rank * s, (self.rank + 1) * s

    @property
    def cols(self) -> tuple[int, int]:
        """Weight columns (x columns) this rank owns."""
        if self.mode == "column":
            return 0, self.k
        s = self.k // self.world
        return self.rank * s, (self.rank + 1) * s

    def shard(self, w: torch.Tensor) -> torch.Tensor:
        r0, r1 = self.rows
        c0, c1 = self.cols
        return w[r0:r1, c0:c1].contiguous()

    def x_slice(self, x: torch.Tensor) -> torch.Tensor:
        c0, c1 = self.cols
        return x if (c0, c1) == (0, self.k) else x[:, c0:c1].contiguous()

    def scatter_cols(self) -> tuple[int, int]:
        """Output columns this rank keeps after a row-parallel reduce-scatter."""
        s = self.n // self.world
        return self.rank * s, (self.rank + 1) * s


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class TPLinear:
    """One tensor-parallel projection on this rank's GPU."""

    def __init__(self, w: torch.Tensor, mode: str, group=None, reduce: str = "all", base_mode: int = BASE_TILE):
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        n, k = w.shape
        self.plan = TPPlan(mode, world, rank, n, k)
        if reduce not in ("all", "scatter"):
            raise ValueError(reduce)
        self.reduce = reduce
        dev = torch.device("cuda", torch.cuda.current_device())
        self.packed: PackedC12 = pack_c12(self.plan.shard(w.to(dev)), base_mode)

    def _local(self, x: torch.Tensor, out_dtype) -> torch.Tensor:
        xs = self.plan.x_slice(x)
        if xs.shape[0] <= GEMV_MAX_M:
            return gemv(self.packed, xs, out_dtype=out_dtype)
        return gemm(self.packed, xs, out_dtype=out_dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        p = self.plan
        m = x.shape[0]
        if p.mode == "column":
            local = self._local(x, torch.bfloat16)                        # [m, n/P]
            if p.world == 1:
                return local
            ns = p.n // p.world
            gathered = torch.empty((p.world * m, ns), dtype=torch.bfloat16, device=x.device)
            dist.all_gather_into_tensor(gathered, local, group=self.group)  # [P][m][ns]
            out = torch.empty((m, p.n), dtype=torch.bfloat16, device=x.device)
            check(lib().mbp_tp_assemble_columns(ctypes.c_void_p(gathered.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                                p.world, m, ns, _stream()), "mbp_tp_assemble_columns")
            return out
        part = self._local(x, torch.float32)                                # [m, n] FP32 partial sums
        if p.world > 1 and self.reduce == "all":
            dist.all_reduce(part, group=self.group)
        elif p.world > 1:
            # reduce-scatter along output columns: transpose-free by scattering a column-major copy's rows
            ns = p.n // p.world
            part_t = part.t().contiguous()                                  # [n, m]
            mine = torch.empty((ns, m), dtype=torch.float32, device=x.device)
            dist.reduce_scatter_tensor(mine, part_t, group=self.group)
            part = mine.t().contiguous()                                    # [m, n/P]
        out = torch.empty(part.shape, dtype=torch.bfloat16, device=x.device)
        check(lib().mbp_f32_to_bf16(ctypes.c_void_p(part.data_ptr()), ctypes.c_void_p(out.data_ptr()), part.numel(),
                                    _stream()), "mbp_f32_to_bf16")
        return out

    __call__ = forward

    @property
    def payload_bytes(self) -> int:
        return self.packed.payload_bytes


DEFAULT_MODES = {"qkv_gate": "column", "o": "row", "pooler": "column", "unpooler": "column"}


def prepare_tp(weights: dict, group=None, modes: dict | None = None, reduce: str = "all") -> dict:
    """``prepare`` for P ranks: every rank passes the full weights; each keeps and packs its shard."""
    modes = dict(DEFAULT_MODES if modes is None else modes)
    return {"tp": {name: TPLinear(w, modes.get(name, "column"), group, reduce) for name, w in weights.items()}}


def kernel_fn_tp(data: dict, state: dict) -> torch.Tensor:
    """``kernel_fn`` for P ranks: the full projection output (all-reduce / all-gather) on every rank."""
    layer = data["config"]["layer"]
    x = data["x"]
    if not x.is_contiguous():
        x = x.contiguous()
    return state["tp"][layer](x)
