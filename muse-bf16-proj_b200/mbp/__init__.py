"""B200-native small-M projection: a drop-in for the reference's ``prepare`` / ``kernel_fn`` API.

Reference (NathenFernandes/muse-bf16-proj, submission.py): types ``Weights`` / ``Config`` / ``Inputs`` (S:21-39),
``prepare(weights) -> state`` (S:7183) and ``kernel_fn(data, state) -> out`` (S:7189).

* ``prepare`` packs every BF16 layer into the lossless 12-bit format on the GPU and the FP32 router into a BF16
  hi/lo pair, checks the packing round trip bit for bit on the device, and returns the state.
* ``kernel_fn`` routes one call to one kernel launch: the weight-streaming GEMV for BF16 layers at m <= 32
  (the reference's decode routes), the tcgen05 verify GEMM at m > 32 (its verify routes), and the hi/lo GEMV
  for the router, writing a NEW output tensor ``[m, n]`` (BF16, FP32 for the router) like the reference
  (README.md:36; S:404, S:889).

Unlike the reference there is no fallback: an unsupported call raises instead of dropping to SGLang.
"""
from __future__ import annotations

from typing import TypedDict

import torch

from . import ops, store
from ._lib import MbpError, device_status, lib, set_wait_limit
from .ops import (BASE_MATRIX, BASE_TILE, PackedC12, PackedHiLo, gemm, gemv, gemv_plan, pack_c12, pack_hilo,
                  router, router_tc, router_topk, unpack_c12)
from .store import load_packed, save_packed

__all__ = ["Weights", "Config", "Inputs", "prepare", "kernel_fn", "MbpError", "PackedC12", "PackedHiLo", "pack_c12",
           "unpack_c12", "pack_hilo", "gemv", "gemm", "gemv_plan", "router", "device_status", "BASE_MATRIX", "BASE_TILE",
           "save_packed", "load_packed", "store", "router_topk", "route", "set_wait_limit", "router_tc"]

LAYERS = ("qkv_gate", "o", "pooler", "unpooler", "router")
GEMV_MAX_M = 32  # the reference's decode/verify boundary: small-M GEMVs up to 32 tokens (SM_MAX_M, S:252)


class Weights(TypedDict):
    qkv_gate: torch.Tensor  # bfloat16 [N, K]
    o: torch.Tensor         # bfloat16 [N, K]
    pooler: torch.Tensor    # bfloat16 [N, K]
    unpooler: torch.Tensor  # bfloat16 [N, K]
    router: torch.Tensor    # float32 [E, K]


class Config(TypedDict):
    m: int
    n: int
    k: int
    layer: str


class Inputs(TypedDict):
    x: torch.Tensor
    config: Config


def prepare(weights: Weights, base_mode: int = BASE_TILE, verify: bool = True, cache: str | None = None) -> dict:
    """Packs every layer on its device.  ``weights`` may hold any subset of the five layers and any shapes with
    rows % 16 == 0 and columns % 64 == 0.  BF16 tensors take the 12-bit path, FP32 tensors the hi/lo path.

    ``cache``: path of a packed weight file (``mbp.store``).  When it holds exactly these layers (same
    fingerprints and base mode) the state is loaded from it instead of packing; otherwise the layers are packed
    (and verified) and the file is written."""
    fps = None
    if cache is not None:
        fps = {name: store.fingerprint(w) for name, w in weights.items()}
        if store.matches(cache, fps, base_mode):
            return store.load_packed(cache, {name: w.device for name, w in weights.items()})
    state: dict = {"layers": {}, "hilo": {}, "k": {}}
    for name, w in weights.items():
        if not isinstance(w, torch.Tensor) or not w.is_cuda:
            raise ValueError(f"layer {name}: expected a CUDA tensor")
        dev = w.device
        with torch.cuda.device(dev):
            if lib().mbp_device_check(dev.index) != 0:
                raise MbpError(-10, f"layer {name} on {dev}")
            if w.dtype == torch.float32:
                state["hilo"][name] = pack_hilo(w)
            elif w.dtype == torch.bfloat16:
                p = pack_c12(w, base_mode)
                if verify and not torch.equal(unpack_c12(p), w):
                    raise RuntimeError(f"layer {name}: 12-bit packing round trip is not exact")
                state["layers"][name] = p
            else:
                raise ValueError(f"layer {name}: unsupported dtype {w.dtype}")
            state["k"][name] = w.shape[1]
    if cache is not None:
        store.save_packed(state, cache, fps, base_mode)
    return state


def kernel_fn(data: Inputs, state: dict) -> torch.Tensor:
    """One projection: ``x @ W[:n].T`` (BF16 out) or the router's FP32 logits."""
    x = data["x"]
    cfg = data["config"]
    layer, n = cfg["layer"], int(cfg["n"])
    if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_cuda:
        raise ValueError("x must be a 2-D bf16 CUDA tensor")
    if not x.is_contiguous():
        x = x.contiguous()
    p = state["layers"].get(layer)
    if p is None:
        if layer in state["hilo"]:
            h = state["hilo"][layer]
            if n != h.n:
                raise ValueError(f"router output width {n} != {h.n}")
            return router(h, x)
        raise KeyError(f"layer {layer!r} was not prepared")
    if not 0 < n <= p.n or n % 16:
        raise ValueError(f"n={n} must be a multiple of 16 in (0, {p.n}]")
    if x.shape[1] != p.k or x.device != p.units.device or x.data_ptr() % 16:
        ops._check_x(x, p.k, p.units.device)  # raises with the reason
    return ops.project(p, x, n, x.shape[0] > GEMV_MAX_M)


def route(data: Inputs, state: dict, k: int, renorm: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """The router call followed by its consumer: ``kernel_fn`` on the router layer, then each token's k experts
    (``router_topk``: ids in descending logit order, softmax weights over the selection or the whole row).  Two
    launches, the second a programmatic dependent of the first."""
    return router_topk(kernel_fn(data, state), k, renorm)
