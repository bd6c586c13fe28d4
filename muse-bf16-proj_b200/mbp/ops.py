"""Device-resident packed weights and the kernel calls behind ``prepare`` / ``kernel_fn``.

Every function here launches hand-written sm_100a CUDA from libmbp.so on the current PyTorch stream; torch is
only used to own device memory.  Nothing falls back to the CPU or to a library GEMM.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from ._lib import C12, Geom, HiLo, check, lib

BASE_MATRIX, BASE_TILE = 0, 1


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device | None = None):
    """The current CUDA stream of `device` (default: the current device) as a raw handle for the C ABI."""
    if _raw_stream is not None:
        return _raw_stream(torch.cuda.current_device() if device is None or device.index is None else device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None):
    return t.data_ptr() if t is not None and t.numel() else None


@dataclass
class PackedC12:
    """A BF16 matrix W[n, k] in the lossless 12-bit format (units, per-tile bases, escape list) on the device."""
    units: torch.Tensor    # uint8 [n/16, k/64, 1536]
    bases: torch.Tensor    # uint8 [n/16]
    esc_off: torch.Tensor  # int32 [(n/16)*(k/64) + 1]
    esc: torch.Tensor      # int32 [n_esc] (bit patterns of uint32 entries)
    n: int
    k: int
    n_esc: int
    desc: C12 = field(init=False, repr=False)

    def __post_init__(self):
        self.desc = C12(self.units.data_ptr(), self.bases.data_ptr(), self.esc_off.data_ptr(),
                        self.esc.data_ptr() if self.n_esc else 0, self.n, self.k, self.n_esc)
        self.desc_ptr = ctypes.pointer(self.desc)  # reused by every call (no per-call ctypes wrapper)

    @property
    def nbytes(self) -> int:
        return self.units.numel() + self.bases.numel() + self.esc_off.numel() * 4 + self.n_esc * 4

    @property
    def payload_bytes(self) -> int:
        """Bytes a full GEMV streams: units + escape entries (the roofline's algorithmic weight bytes)."""
        return self.units.numel() + self.n_esc * 4

    @property
    def dense_escapes(self) -> bool:
        """At least one escape per 1000 weights (the GEMV planner's dense class)."""
        return self.n_esc * 1000 >= self.n * self.k

    def plan(self, m: int, n_out: int | None = None, f32_out: bool = False) -> Geom:
        """The geometry `gemv(self, x)` launches with for m tokens."""
        return gemv_plan(self.n if n_out is None else n_out, self.k, m, self.n_esc > 0, f32_out, self.dense_escapes)


@dataclass
class PackedHiLo:
    """An FP32 matrix as a BF16 hi/lo pair of uncompressed units [n/16, k/64, 2, 2048] on the device."""
    units: torch.Tensor
    n: int
    k: int
    desc: HiLo = field(init=False, repr=False)

    def __post_init__(self):
        self.desc = HiLo(self.units.data_ptr(), self.n, self.k)

    @property
    def payload_bytes(self) -> int:
        return self.units.numel()


def project(p: PackedC12, x: torch.Tensor, n_out: int, tensor_cores: bool) -> torch.Tensor:
    """The per-call fast path of ``kernel_fn``: a new BF16 [m, n_out] output from the GEMV or the tcgen05 GEMM.
    The caller has checked x (contiguous BF16 [m, k] CUDA tensor on the weights' device) and n_out."""
    m = x.shape[0]
    dev = x.device
    out = torch.empty((m, n_out), dtype=torch.bfloat16, device=dev)
    L = lib()
    if tensor_cores:
        rc = L.mbp_gemm_c12(p.desc_ptr, x.data_ptr(), m, n_out, out.data_ptr(), n_out, _stream(dev))
    else:
        rc = L.mbp_gemv_c12(p.desc_ptr, x.data_ptr(), m, n_out, out.data_ptr(), n_out, None, _stream(dev))
    if rc:
        check(rc, "mbp_gemm_c12" if tensor_cores else "mbp_gemv_c12")
    return out


def _check_weight(w: torch.Tensor, dtype) -> None:
    if not w.is_cuda or w.dtype != dtype or w.dim() != 2:
        raise ValueError(f"expected a 2-D {dtype} CUDA tensor, got {w.dtype} {tuple(w.shape)} on {w.device}")
    n, k = w.shape
    if n % 16 or k % 64:
        raise ValueError(f"weight shape {tuple(w.shape)}: rows must be a multiple of 16, columns of 64")


def pack_c12(w: torch.Tensor, base_mode: int = BASE_TILE) -> PackedC12:
    """GPU packer (replaces the reference's host packer, submission.py S:82-227)."""
    _check_weight(w, torch.bfloat16)
    w = w.contiguous()
    n, k = w.shape
    r, c = n // 16, k // 64
    dev = w.device
    L = lib()
    units = torch.empty((r, c, 1536), dtype=torch.uint8, device=dev)
    bases = torch.empty(r, dtype=torch.uint8, device=dev)
    esc_off = torch.empty(r * c + 1, dtype=torch.int32, device=dev)
    ws_bytes = L.mbp_pack_c12_workspace(n, k)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    st = _stream()
    check(L.mbp_pack_c12(_ptr(w), n, k, base_mode, _ptr(units), _ptr(bases), _ptr(esc_off), _ptr(ws), ws_bytes, st),
          "mbp_pack_c12")
    n_esc = int(esc_off[-1].item())
    esc = torch.empty(max(n_esc, 0), dtype=torch.int32, device=dev)
    check(L.mbp_pack_c12_escapes(_ptr(w), n, k, _ptr(bases), _ptr(esc_off), _ptr(esc) if n_esc else None, st),
          "mbp_pack_c12_escapes")
    return PackedC12(units, bases, esc_off, esc, n, k, n_esc)


def unpack_c12(p: PackedC12) -> torch.Tensor:
    out = torch.empty((p.n, p.k), dtype=torch.bfloat16, device=p.units.device)
    check(lib().mbp_unpack_c12(ctypes.byref(p.desc), _ptr(out), _stream()), "mbp_unpack_c12")
    return out


def pack_hilo(w: torch.Tensor) -> PackedHiLo:
    """FP32 -> BF16 hi/lo units (replaces pack_router, S:876-879)."""
    _check_weight(w, torch.float32)
    w = w.contiguous()
    n, k = w.shape
    units = torch.empty((n // 16, k // 64, 2, 2048), dtype=torch.uint8, device=w.device)
    check(lib().mbp_pack_hilo(_ptr(w), n, k, _ptr(units), _stream()), "mbp_pack_hilo")
    return PackedHiLo(units, n, k)


PLAN_ESCAPES, PLAN_F32_OUT, PLAN_DENSE_ESCAPES = 1, 2, 4


def gemv_plan(n_out: int, k: int, m: int, escapes: bool = True, f32_out: bool = False, dense: bool = False) -> Geom:
    """The launch geometry the GEMV uses for this shape when no geometry is given (`dense`: at least one escape
    per 1000 weights)."""
    g = Geom()
    flags = ((PLAN_ESCAPES if escapes or dense else 0) | (PLAN_F32_OUT if f32_out else 0)
             | (PLAN_DENSE_ESCAPES if dense else 0))
    check(lib().mbp_gemv_plan_ex(n_out, k, m, flags, ctypes.byref(g)), "mbp_gemv_plan_ex")
    return g


def _check_x(x: torch.Tensor, k: int, device) -> None:
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != k or not x.is_cuda:
        raise ValueError(f"x must be a CUDA bf16 [m, {k}] tensor, got {x.dtype} {tuple(x.shape)}")
    if x.device != device:
        raise ValueError(f"x on {x.device}, weights on {device}")
    if not x.is_contiguous() or x.data_ptr() % 16:
        raise ValueError("x must be contiguous and 16-byte aligned")


def gemv(p: PackedC12, x: torch.Tensor, n_out: int | None = None, out: torch.Tensor | None = None,
         out_dtype=torch.bfloat16, geom: Geom | None = None) -> torch.Tensor:
    """out[m, n_out] = x . W[:n_out]^T through the weight-streaming GEMV."""
    n_out = p.n if n_out is None else n_out
    _check_x(x, p.k, p.units.device)
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n_out), dtype=out_dtype, device=x.device)
    if out.dim() != 2 or out.shape[0] != m or out.shape[1] < n_out or out.stride(1) != 1:
        raise ValueError("bad out tensor")
    fn = lib().mbp_gemv_c12_f32 if out.dtype == torch.float32 else lib().mbp_gemv_c12
    if out.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"unsupported output dtype {out.dtype}")
    check(fn(ctypes.byref(p.desc), x.data_ptr(), m, n_out, out.data_ptr(), out.stride(0),
             ctypes.byref(geom) if geom is not None else None, _stream(x.device)), "mbp_gemv_c12")
    return out


def gemm(p: PackedC12, x: torch.Tensor, n_out: int | None = None, out: torch.Tensor | None = None,
         out_dtype=torch.bfloat16) -> torch.Tensor:
    """out[m, n_out] = x . W[:n_out]^T through the tcgen05 verify GEMM (replaces S:783/979/1547/2985)."""
    n_out = p.n if n_out is None else n_out
    _check_x(x, p.k, p.units.device)
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n_out), dtype=out_dtype, device=x.device)
    if out.dim() != 2 or out.shape[0] != m or out.shape[1] < n_out or out.stride(1) != 1:
        raise ValueError("bad out tensor")
    if out.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"unsupported output dtype {out.dtype}")
    fn = lib().mbp_gemm_c12_f32 if out.dtype == torch.float32 else lib().mbp_gemm_c12
    check(fn(ctypes.byref(p.desc), x.data_ptr(), m, n_out, out.data_ptr(), out.stride(0), _stream(x.device)),
          "mbp_gemm_c12")
    return out


def router(p: PackedHiLo, x: torch.Tensor, out: torch.Tensor | None = None, geom: Geom | None = None):
    """out_f32[m, n] = x . (hi + lo)^T (replaces rr_launch / rr_scalar / rr_small, S:856-861)."""
    _check_x(x, p.k, p.units.device)
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, p.n), dtype=torch.float32, device=x.device)
    check(lib().mbp_router_hilo(ctypes.byref(p.desc), x.data_ptr(), m, out.data_ptr(), out.stride(0),
                                ctypes.byref(geom) if geom is not None else None, _stream(x.device)),
          "mbp_router_hilo")
    return out


def router_tc(p: PackedHiLo, x: torch.Tensor, out: torch.Tensor | None = None, bn: int = 0, split: int = 0):
    """The router product on the tcgen05 tensor cores (``router`` takes this path above 256 tokens): token tile
    ``bn`` (multiple of 16, <= 128) and K split over a cluster of ``split`` CTAs (<= 16, and at least k / 2048:
    no CTA accumulates more than 2048 columns on the tensor pipe, which keeps the 1e-5 accuracy); 0 chooses."""
    _check_x(x, p.k, p.units.device)
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, p.n), dtype=torch.float32, device=x.device)
    if out.dtype != torch.float32 or out.dim() != 2 or out.shape != (m, p.n) or out.stride(1) != 1:
        raise ValueError("out must be a float32 [m, n] tensor with unit column stride")
    check(lib().mbp_router_hilo_tc(ctypes.byref(p.desc), x.data_ptr(), m, out.data_ptr(), out.stride(0), bn, split,
                                   _stream(x.device)), "mbp_router_hilo_tc")
    return out


def router_topk(logits: torch.Tensor, k: int, renorm: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """(weights f32 [m, k], ids int32 [m, k]): each row's k largest logits in descending order (equal logits:
    lower index first) and their softmax weights over the selection (renorm) or over the whole row."""
    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_cuda or logits.stride(1) != 1:
        raise ValueError("logits must be a CUDA float32 [m, e] tensor with unit column stride")
    m, e = logits.shape
    w = torch.empty((m, k), dtype=torch.float32, device=logits.device)
    ids = torch.empty((m, k), dtype=torch.int32, device=logits.device)
    check(lib().mbp_router_topk(_ptr(logits), m, e, logits.stride(0), k, int(bool(renorm)), _ptr(w), _ptr(ids),
                                _stream()), "mbp_router_topk")
    return w, ids
