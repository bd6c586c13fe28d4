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

**Peer-store transport** (``transport="p2p"``, the default on one node, used for the GEMV calls m <= 32): instead
of a GEMV, an NCCL collective and an assembly kernel, ONE kernel per call (``mbp_gemv_c12_tp``): the GEMV stores
its results straight into every rank's exchange buffer over NVLink (buffers mapped through CUDA IPC, plain
stores, no multicast) as 64-bit words whose upper half is the exchange's epoch, and then each CTA waits until
the words of its own tiles from every rank carry the epoch and writes them to the output: column-parallel, rank
r's GEMV writes its column block of the [m, N] output into every rank's buffer and each CTA gathers its tiles'
columns of all ranks; row-parallel, rank r writes its FP32 partial into slot r of every rank's [P, m, N] buffer
and each CTA adds its tiles' P slots in rank order (the same order, hence the same bits, on every rank) into
BF16.  A word and its tag arrive in one store, so no system-scope fence (several microseconds each) is needed.
Each layer has two exchange buffers, picked by the parity of an epoch counter kept in device memory (the grid's
last CTA advances it), so back-to-back calls and CUDA-graph replays never write a buffer a peer may still be
reading.  ``fused=False`` (or a shard geometry whose grid cannot be resident all at once) runs the GEMV
(``mbp_gemv_c12_multi``) and then a separate receive kernel (``mbp_tp_finish``) over the same words.  The GEMM
calls (m > 32) and ``reduce="scatter"`` keep the NCCL path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ._lib import (OUT_TAGGED_BF16X2, OUT_TAGGED_F32, TP_BARRIER, TP_COUNTER_SLOTS, TP_GATHER_BF16, TP_RSAG, TP_SUM_F32,
                   TPExchange, check, lib)
from .ops import BASE_TILE, PackedC12, gemm, gemv, pack_c12

GEMV_MAX_M = 32
GEMM_EXCHANGE_MAX_M = 256  # column-parallel GEMM calls up to this size exchange by peer stores (buffers sized for it)
_ERR_SPLIT = -3  # MBP_ERR_SPLIT


# ---------------- device memory exchanged between the ranks of a node ----------------

class PeerBuffer:
    """One zeroed device buffer per rank of `group`, each mapped into every rank (CUDA IPC); ``ptrs[r]`` is rank
    r's buffer as seen from this process."""

    def __init__(self, nbytes: int, group=None):
        self.group, self.nbytes = group, nbytes
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        check(lib().mbp_ipc_alloc(nbytes, ctypes.byref(own), handle), "mbp_ipc_alloc")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.own = own.value
        self.ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            check(lib().mbp_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)), "mbp_ipc_open")
            self.ptrs.append(p.value)

    def local_first(self, offset: int = 0):
        """Pointers (plus a byte offset) with this rank's first, as a ctypes array for mbp_gemv_c12_multi."""
        order = [self.rank] + [r for r in range(self.world) if r != self.rank]
        return (ctypes.c_void_p * self.world)(*[self.ptrs[r] + offset for r in order])

    @property
    def closed(self) -> bool:
        return self.own is None

    def close(self):
        """Collective over the group (every rank calls it, in the same order as its other collectives): waits for
        this device's queued work, unmaps the peers' buffers once every rank has got that far, and frees this
        rank's own buffer once every rank has unmapped it.  A second call does nothing."""
        if self.own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)        # no rank's kernels still store into or read from any buffer
        for r, ptr in enumerate(self.ptrs):
            if r != self.rank:
                check(lib().mbp_ipc_close(ctypes.c_void_p(ptr)), "mbp_ipc_close")
        dist.barrier(group=self.group)        # every peer mapping of this rank's buffer is gone
        own, self.own, self.ptrs = self.own, None, []
        check(lib().mbp_ipc_free(ctypes.c_void_p(own)), "mbp_ipc_free")


class _GroupSync:
    """Exchange state of one process group: every rank's flag array (peer-mapped) and this rank's epoch slots,
    shared by all peer-store layers of the group (every rank makes the same sequence of exchanges)."""

    def __init__(self, group=None):
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.flags = PeerBuffer(64, group)
        # epoch slots + the fused GEMV's grid ticket
        self.counter = torch.zeros(TP_COUNTER_SLOTS + 1, dtype=torch.int32,
                                   device=torch.device("cuda", torch.cuda.current_device()))
        self.flag_ptrs = (ctypes.c_void_p * self.world)(*self.flags.ptrs)

    def finish(self, buf: PeerBuffer | None, parity_stride: int, mode: int, m: int, n: int,
               out: torch.Tensor | None):
        check(lib().mbp_tp_finish(self.flag_ptrs, self.rank, self.world, ctypes.c_void_p(self.counter.data_ptr()),
                                  ctypes.c_void_p(buf.own if buf else 0), parity_stride, mode, m, n,
                                  ctypes.c_void_p(out.data_ptr() if out is not None else 0), _stream()),
              "mbp_tp_finish")

    def barrier(self):
        """Flag barrier of the group on the current stream (orders every rank's earlier stores before it)."""
        self.finish(None, 0, TP_BARRIER, 0, 0, None)

    def close(self):
        """Collective: releases the flag arrays (see ``PeerBuffer.close``)."""
        self.flags.close()


def _p2p_placement_ok(seen: list, host: str, local: dict, dev: int, can_access) -> bool:
    """The peer-store rule for one rank: `seen` = (hostname, GPU uuid) of every rank, `local` = uuid -> device
    index of the GPUs this process sees, `dev` = this rank's device index, `can_access(a, b)` = peer access.
    True only for at most 8 ranks on this host, each on a GPU of its own (waiting kernels of two ranks on one GPU
    are not guaranteed to run at the same time), every peer's GPU visible to this process and peer-accessible
    from this rank's GPU.  A peer this process cannot see (per-rank device lists) gives False: whether its
    exchange buffer could be mapped through CUDA IPC is then unknown, and NCCL needs no such mapping."""
    if len(seen) > 8 or len({u for _, u in seen}) != len(seen) or any(h != host for h, _ in seen):
        return False
    if any(u not in local for _, u in seen):
        return False
    return all(can_access(dev, local[u]) for _, u in seen if local[u] != dev)


def _same_node(group) -> bool:
    """True when every rank of `group` drives a different GPU of this host and all pairs are peer-capable (the
    exchange's waits need the ranks on separate GPUs running concurrently); every rank must agree."""
    import socket
    world = dist.get_world_size(group)
    dev = torch.cuda.current_device()
    me = (socket.gethostname(), str(torch.cuda.get_device_properties(dev).uuid))
    seen = [None] * world
    dist.all_gather_object(seen, me, group=group)
    # peers visible to this process by uuid (all of them when ranks share the device list)
    local = {str(torch.cuda.get_device_properties(i).uuid): i for i in range(torch.cuda.device_count())}
    ok = _p2p_placement_ok([tuple(s) for s in seen], me[0], local, dev, torch.cuda.can_device_access_peer)
    votes = [None] * world
    dist.all_gather_object(votes, ok, group=group)
    return all(votes)


_SYNCS: dict = {}


def _sync_key(group):
    return id(group) if group is not None else None


def _group_sync(group) -> _GroupSync:
    key = _sync_key(group)
    if key not in _SYNCS:
        _SYNCS[key] = _GroupSync(group)
    return _SYNCS[key]


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


def exchange_route(mode: str, reduce: str, world: int, m: int, peer_buffers: bool) -> str:
    """How a call of `m` tokens exchanges: "gemv-p2p" (the GEMV's tagged peer stores, m <= 32), "gemm-p2p" (the
    tcgen05 GEMM's tagged peer stores: column-parallel up to 256 tokens, row-parallel ones at 2 ranks) or "nccl"
    (everything else, and every call of a layer without peer buffers)."""
    if not peer_buffers or m < 1:
        return "nccl"
    if m <= GEMV_MAX_M:
        return "gemv-p2p" if mode == "column" or reduce == "all" else "nccl"
    if m <= GEMM_EXCHANGE_MAX_M and (mode == "column" or (reduce == "all" and world == 2)):
        return "gemm-p2p"
    return "nccl"


def row_exchange_for(world: int, requested: str = "auto") -> str:
    """The fused row-parallel exchange a layer of `world` ranks uses: "sum" (every rank's FP32 partial to every
    rank) or "rsag" (reduce-scatter to each tile's owner + BF16 gather); "auto" = "rsag" from 4 ranks on."""
    if requested not in ("auto", "sum", "rsag"):
        raise ValueError(f"row_exchange must be auto, sum or rsag, got {requested!r}")
    if requested != "auto":
        return requested
    return "rsag" if world >= 4 else "sum"


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class TPLinear:
    """One tensor-parallel projection on this rank's GPU.

    ``transport``: "p2p" stores GEMV results straight into the peers' exchange buffers (one node, every pair of
    GPUs peer-capable), "nccl" runs the GEMV then an NCCL collective, "auto" picks "p2p" when the group spans
    more than one GPU of this node and NCCL otherwise (p2p also carries the column-parallel GEMM calls up to
    256 tokens; the row-parallel GEMM calls, m > 32, use NCCL).
    ``fused`` (p2p): one kernel per call (``mbp_gemv_c12_tp``: the GEMV's CTAs also wait for and assemble their
    tiles from the other ranks); False runs the GEMV and then the separate receive kernel (``mbp_tp_finish``).
    ``row_exchange`` (p2p, row-parallel, fused): "sum" sends every rank's FP32 partial to every rank; "rsag" sends
    each tile's partials to one owner rank, which adds them and sends the BF16 result to all (reduce-scatter +
    gather: (P-1)/P x 12 m n bytes per rank instead of (P-1) x 8 m n); "auto" = "rsag" from 4 ranks on.  Both
    give the same bits (rank-order FP32 sums)."""

    def __init__(self, w: torch.Tensor, mode: str, group=None, reduce: str = "all", base_mode: int = BASE_TILE,
                 transport: str = "auto", fused: bool = True, row_exchange: str = "auto"):
        self.fused = fused
        self._two_kernel_m: set = set()
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        n, k = w.shape
        self.plan = TPPlan(mode, world, rank, n, k)
        if reduce not in ("all", "scatter"):
            raise ValueError(reduce)
        if transport not in ("auto", "p2p", "nccl"):
            raise ValueError(transport)
        self.reduce = reduce
        self.row_exchange = row_exchange_for(world, row_exchange)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.packed: PackedC12 = pack_c12(self.plan.shard(w.to(dev)), base_mode)
        if transport == "auto":
            transport = "p2p" if world > 1 and _same_node(group) else "nccl"
        self.transport = transport
        self._xbuf: PeerBuffer | None = None
        if transport == "p2p" and world > 1:
            self._setup_p2p(dev)

    def _setup_p2p(self, dev):
        p = self.plan
        # exchange buffers of epoch-tagged 64-bit words, two per rank (epoch parity)
        if p.mode == "column":
            per = GEMM_EXCHANGE_MAX_M * (p.n // 2) * 8                       # [m_max][n/2] bf16-pair words
        else:
            per = p.world * GEMV_MAX_M * p.n * 8                             # [P][m_max][n] f32 words
            per += GEMV_MAX_M * (p.n // 2) * 8                               # + the reduce-scatter's gather region
            if self._gemm_row_p2p():
                per = max(per, p.world * GEMM_EXCHANGE_MAX_M * p.n * 8)      # the GEMM calls' [P][m][n] partials
        self._sync = _group_sync(self.group)
        self._par = -(-per // 256) * 256                                       # parity-1 buffer offset
        self._xbuf = PeerBuffer(2 * self._par, self.group)
        ex = TPExchange()
        for r, ptr in enumerate(self._xbuf.ptrs):
            ex.bufs[r] = ptr
        ex.parity_stride = self._par
        ex.counter = self._sync.counter.data_ptr()
        ex.rank, ex.P, ex.n = p.rank, p.world, p.n
        ex.mode = (TP_GATHER_BF16 if p.mode == "column" else
                   TP_RSAG if self.row_exchange == "rsag" else TP_SUM_F32)
        self._ex = ex

    def _forward_p2p(self, x: torch.Tensor) -> torch.Tensor:
        p = self.plan
        m = x.shape[0]
        out = torch.empty((m, p.n), dtype=torch.bfloat16, device=x.device)
        if self.fused and m not in self._two_kernel_m:
            # one kernel: the shard's GEMV stores into every rank's buffer and each CTA assembles its tiles
            xp = x.data_ptr() + (0 if p.mode == "column" else p.rank * (p.k // p.world) * 2)
            rc = lib().mbp_gemv_c12_tp(ctypes.byref(self.packed.desc), ctypes.c_void_p(xp), p.k, m,
                                       ctypes.byref(self._ex), ctypes.c_void_p(out.data_ptr()), None, _stream())
            if rc != _ERR_SPLIT:
                check(rc, "mbp_gemv_c12_tp")
                return out
            # this shard's geometry cannot have its whole grid resident at once (every rank plans the same
            # geometry, so every rank takes this branch): the GEMV and the separate receive kernel, which use
            # the same words, buffers and epochs
            self._two_kernel_m.add(m)
        buf, sync = self._xbuf, self._sync
        epoch = ctypes.c_void_p(sync.counter.data_ptr())
        if p.mode == "column":
            # this rank's rows [r*ns, (r+1)*ns) are word columns [r*ns/2, (r+1)*ns/2) of every rank's buffer
            ns = p.n // p.world
            check(lib().mbp_gemv_c12_multi(ctypes.byref(self.packed.desc), ctypes.c_void_p(x.data_ptr()), p.k, m, ns,
                                           buf.local_first(p.rank * (ns // 2) * 8), p.world, p.n // 2,
                                           OUT_TAGGED_BF16X2, epoch, self._par, None, _stream()),
                  "mbp_gemv_c12_multi")
            sync.finish(buf, self._par, TP_GATHER_BF16, m, p.n, out)
            return out
        # this rank's FP32 partial of all n outputs from its K slice goes to slot r of every rank's buffer
        ks = p.k // p.world
        check(lib().mbp_gemv_c12_multi(ctypes.byref(self.packed.desc), ctypes.c_void_p(x.data_ptr() + p.rank * ks * 2),
                                       p.k, m, p.n, buf.local_first(p.rank * m * p.n * 8), p.world, p.n,
                                       OUT_TAGGED_F32, epoch, self._par, None, _stream()), "mbp_gemv_c12_multi")
        sync.finish(buf, self._par, TP_SUM_F32, m, p.n, out)
        return out

    def _gemm_row_p2p(self) -> bool:
        """Row-parallel GEMM calls exchange their FP32 partials by peer stores at 2 ranks only (`exchange_route`):
        every rank sends its whole [m][n] partial to every rank, (P-1) x 8 m n bytes, which beats NCCL's
        all-reduce at P = 2 but not beyond (at 256 tokens and P = 8, 88 MB per rank)."""
        return self.plan.mode == "row" and self.plan.world == 2

    def _forward_gemm_p2p(self, x: torch.Tensor) -> torch.Tensor:
        """A call above 32 tokens through the tcgen05 GEMM's peer stores.  Column-parallel: the shard's result as
        tagged bf16x2 words into every rank's buffer (its columns of the [m][n/2] word grid), assembled by the
        receive kernel.  Row-parallel (2 ranks): the shard's FP32 partial of all n outputs as tagged f32 words
        into slot `rank` of every rank's buffer, summed in rank order and rounded by the receive kernel.  Same
        words, epochs and parity halves as the GEMV calls."""
        p = self.plan
        m = x.shape[0]
        out = torch.empty((m, p.n), dtype=torch.bfloat16, device=x.device)
        sync = self._sync
        epoch = ctypes.c_void_p(sync.counter.data_ptr())
        if p.mode == "column":
            ns = p.n // p.world
            check(lib().mbp_gemm_c12_multi(ctypes.byref(self.packed.desc), ctypes.c_void_p(x.data_ptr()), m, ns,
                                           self._xbuf.local_first(p.rank * (ns // 2) * 8), p.world, p.n // 2,
                                           OUT_TAGGED_BF16X2, epoch, self._par, _stream()), "mbp_gemm_c12_multi")
            sync.finish(self._xbuf, self._par, TP_GATHER_BF16, m, p.n, out)
            return out
        xs = p.x_slice(x)  # this rank's K columns, contiguous for the GEMM's x tiles
        check(lib().mbp_gemm_c12_multi(ctypes.byref(self.packed.desc), ctypes.c_void_p(xs.data_ptr()), m, p.n,
                                       self._xbuf.local_first(p.rank * m * p.n * 8), p.world, p.n,
                                       OUT_TAGGED_F32, epoch, self._par, _stream()), "mbp_gemm_c12_multi")
        sync.finish(self._xbuf, self._par, TP_SUM_F32, m, p.n, out)
        return out

    def _local(self, x: torch.Tensor, out_dtype) -> torch.Tensor:
        xs = self.plan.x_slice(x)
        if xs.shape[0] <= GEMV_MAX_M:
            return gemv(self.packed, xs, out_dtype=out_dtype)
        return gemm(self.packed, xs, out_dtype=out_dtype)

    def close(self):
        """Collective over the group: releases this layer's exchange buffers and packed shard; later calls raise.
        The group's flag arrays and epoch slots stay (other layers share them; ``release_tp`` drops them)."""
        if self._xbuf is not None:
            self._xbuf.close()
        self._xbuf, self.packed = None, None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.packed is None:
            raise RuntimeError("TPLinear used after close()")
        p = self.plan
        m = x.shape[0]
        route = exchange_route(p.mode, self.reduce, p.world, m, self._xbuf is not None)
        if route != "nccl":
            if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != p.k or not x.is_contiguous():
                raise ValueError(f"x must be a contiguous bf16 [m, {p.k}] tensor")
            if x.device != self.packed.units.device:
                raise ValueError("x is not on this rank's device")
            return self._forward_gemm_p2p(x) if route == "gemm-p2p" else self._forward_p2p(x)
        if p.mode == "column":
            local = self._local(x, torch.bfloat16)                        # [m, n/P]
            if p.world == 1:
                return local
            ns = p.n // p.world
            gathered = torch.empty((p.world * m, ns), dtype=torch.bfloat16, device=x.device)
            dist.all_gather_into_tensor(gathered, local, group=self.group)  # [P][m][ns]
            return self._assemble(gathered, m, ns)
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
        return self._to_bf16(part)

    def _assemble(self, gathered: torch.Tensor, m: int, ns: int) -> torch.Tensor:
        """[P][m][ns] gathered shard outputs -> [m, n] (the NCCL column path's assembly kernel)."""
        out = torch.empty((m, self.plan.n), dtype=torch.bfloat16, device=gathered.device)
        check(lib().mbp_tp_assemble_columns(ctypes.c_void_p(gathered.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                            self.plan.world, m, ns, _stream()), "mbp_tp_assemble_columns")
        return out

    def _to_bf16(self, part: torch.Tensor) -> torch.Tensor:
        """Summed FP32 partials -> BF16 (the NCCL row path's rounding kernel)."""
        out = torch.empty(part.shape, dtype=torch.bfloat16, device=part.device)
        check(lib().mbp_f32_to_bf16(ctypes.c_void_p(part.data_ptr()), ctypes.c_void_p(out.data_ptr()), part.numel(),
                                    _stream()), "mbp_f32_to_bf16")
        return out

    __call__ = forward

    @property
    def payload_bytes(self) -> int:
        return self.packed.payload_bytes


DEFAULT_MODES = {"qkv_gate": "column", "o": "row", "pooler": "column", "unpooler": "column"}


def prepare_tp(weights: dict, group=None, modes: dict | None = None, reduce: str = "all",
               transport: str = "auto") -> dict:
    """``prepare`` for P ranks: every rank passes the full weights; each keeps and packs its shard."""
    modes = dict(DEFAULT_MODES if modes is None else modes)
    return {"tp": {name: TPLinear(w, modes.get(name, "column"), group, reduce, transport=transport)
                   for name, w in weights.items()}}


def release_tp(state: dict):
    """Collective teardown of ``prepare_tp``'s state (every rank of the layers' group calls it with the state it
    prepared): closes every layer in name order, then the flag arrays and epoch slots of the groups those layers
    exchanged over (in the order the names first reach them, the same on every rank)."""
    layers = state.get("tp", {})
    keys = []
    for name in sorted(layers):
        layer = layers[name]
        if layer._xbuf is not None and _sync_key(layer.group) not in keys:
            keys.append(_sync_key(layer.group))
        layer.close()
    for key in keys:
        sync = _SYNCS.pop(key, None)
        if sync is not None:
            sync.close()


def check_exchange(clear: bool = True) -> None:
    """Raises ``MbpError`` when a bounded wait of a peer-store exchange on this device gave up since the last
    check (device status MBP_DEV_TIMEOUT_PEER: a peer's words or flags did not arrive within the wait limit, so
    the outputs of the calls since then may hold stale or partial data).  The kernels never trap and the calls
    themselves do not synchronise, so a caller that needs the guarantee calls this after synchronising a step
    (``torch.cuda.synchronize()``), e.g. once per decode step or after a graph replay."""
    from ._lib import DEVICE_STATUS, MbpError, device_status
    st = device_status(clear)
    if st:
        raise MbpError(-200 - st, f"device status {st} ({DEVICE_STATUS.get(st, 'unknown')})")


def kernel_fn_tp(data: dict, state: dict) -> torch.Tensor:
    """``kernel_fn`` for P ranks: the full projection output (all-reduce / all-gather) on every rank.  Exchange
    failures surface through the device status word, not here: see ``check_exchange``."""
    layer = data["config"]["layer"]
    x = data["x"]
    if not x.is_contiguous():
        x = x.contiguous()
    return state["tp"][layer](x)
