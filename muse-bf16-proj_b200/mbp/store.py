"""Packed on-disk format: the state ``prepare`` builds, saved once and loaded later without packing again.

The reference packs on the host inside ``prepare`` on every start (53.8 s cold for its five layers,
results/v18.json:15).  This build packs on the GPU, and this module keeps the result: a file holds every layer's
device arrays exactly as the kernels read them, so loading is one file read and one host-to-device copy per
array.

File layout (little-endian):

    bytes 0-7       magic b"MBPPACK1"
    bytes 8-15      uint64 H, the length of the JSON header
    bytes 16-16+H   JSON header: {"version": 1, "layers": {name: {"kind": "c12" | "hilo", "n", "k", "n_esc",
                    "base_mode", "fingerprint", "arrays": {array: [offset, nbytes, dtype, shape]}}}}
    then            each array's bytes at its offset (4096-aligned)

c12 layers store ``units`` (uint8 [n/16, k/64, 1536]), ``bases`` (uint8 [n/16]), ``esc_off`` (int32
[(n/16)(k/64)+1]) and ``esc`` (int32 [n_esc]); hi/lo layers store ``units`` (uint8 [n/16, k/64, 2, 2048]).
A layer's fingerprint hashes its source weights' shape, dtype, a fixed strided sample of their bits and two sums
over all of their bits; ``prepare(weights, cache=path)`` re-packs (and rewrites the file) when any fingerprint,
layer set or base mode differs.  The fingerprint tells weight files apart; it is not a proof that every bit
matches.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct

import numpy as np
import torch

from .ops import PackedC12, PackedHiLo

MAGIC = b"MBPPACK1"
VERSION = 1
_ALIGN = 4096
_DT = {"uint8": (np.uint8, torch.uint8), "int32": (np.int32, torch.int32)}


def fingerprint(w: torch.Tensor) -> str:
    """Hash of a weight tensor's shape, dtype, a strided sample of its bits and two sums over all of its bits."""
    bits = w.detach().contiguous().view(torch.int32 if w.dtype == torch.float32 else torch.int16).reshape(-1)
    step = max(1, bits.numel() // 65536)
    sample = bits[::step].cpu().numpy().tobytes()
    total = int(bits.sum(dtype=torch.int64).item())
    odd = int(bits[1::2].sum(dtype=torch.int64).item()) if bits.numel() > 1 else 0
    h = hashlib.sha256()
    h.update(repr((tuple(w.shape), str(w.dtype), total, odd)).encode())
    h.update(sample)
    return h.hexdigest()


def _arrays(p) -> dict:
    if isinstance(p, PackedC12):
        return {"units": p.units, "bases": p.bases, "esc_off": p.esc_off, "esc": p.esc}
    return {"units": p.units}


def save_packed(state: dict, path: str, fingerprints: dict | None = None, base_mode: int | None = None) -> None:
    """Writes every layer of a ``prepare`` state to `path` (atomically: a temporary file is renamed)."""
    layers = {}
    blobs = []
    offset = 0
    items = [(n, p) for n, p in state["layers"].items()] + [(n, p) for n, p in state["hilo"].items()]
    for name, p in items:
        meta = {"kind": "c12" if isinstance(p, PackedC12) else "hilo", "n": p.n, "k": p.k,
                "n_esc": int(getattr(p, "n_esc", 0)), "base_mode": base_mode,
                "fingerprint": (fingerprints or {}).get(name), "arrays": {}}
        for an, t in _arrays(p).items():
            a = t.detach().contiguous().cpu().numpy()
            dt = "uint8" if a.dtype == np.uint8 else "int32"
            meta["arrays"][an] = [offset, int(a.nbytes), dt, list(a.shape)]
            blobs.append((offset, a))
            offset += -(-a.nbytes // _ALIGN) * _ALIGN
        layers[name] = meta
    header = json.dumps({"version": VERSION, "layers": layers}).encode()
    data0 = -(-(16 + len(header)) // _ALIGN) * _ALIGN
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC + struct.pack("<Q", len(header)) + header)
        for off, a in blobs:
            f.seek(data0 + off)
            f.write(a.tobytes())
        f.truncate(data0 + offset)
    os.replace(tmp, path)


def read_header(path: str) -> tuple[dict, int]:
    """(header, byte offset of the array data) of a packed file; raises ValueError if it is not one."""
    with open(path, "rb") as f:
        head = f.read(16)
        if len(head) != 16 or head[:8] != MAGIC:
            raise ValueError(f"{path}: not a packed weight file")
        (hl,) = struct.unpack("<Q", head[8:])
        header = json.loads(f.read(hl))
    if header.get("version") != VERSION:
        raise ValueError(f"{path}: format version {header.get('version')} (this build reads {VERSION})")
    return header, -(-(16 + hl) // _ALIGN) * _ALIGN


def load_packed(path: str, device=None) -> dict:
    """The ``prepare`` state stored in `path`, its arrays on `device` (a device, a {layer: device} mapping, or
    by default the current CUDA device)."""
    header, data0 = read_header(path)
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    state: dict = {"layers": {}, "hilo": {}, "k": {}}
    with open(path, "rb") as f:
        for name, meta in header["layers"].items():
            dev = device[name] if isinstance(device, dict) else device
            ts = {}
            for an, (off, nbytes, dt, shape) in meta["arrays"].items():
                npdt, _ = _DT[dt]
                f.seek(data0 + off)
                a = np.frombuffer(f.read(nbytes), dtype=npdt).reshape(shape)
                if a.nbytes != nbytes:
                    raise ValueError(f"{path}: layer {name} array {an} is truncated")
                ts[an] = torch.from_numpy(a.copy()).to(dev)
            if meta["kind"] == "c12":
                state["layers"][name] = PackedC12(ts["units"], ts["bases"], ts["esc_off"], ts["esc"], meta["n"],
                                                  meta["k"], meta["n_esc"])
            else:
                state["hilo"][name] = PackedHiLo(ts["units"], meta["n"], meta["k"])
            state["k"][name] = meta["k"]
    return state


def matches(path: str, fingerprints: dict, base_mode: int) -> bool:
    """True when `path` is a packed file of exactly these layers, fingerprints and base mode."""
    try:
        header, _ = read_header(path)
    except (OSError, ValueError):
        return False
    layers = header["layers"]
    if set(layers) != set(fingerprints):
        return False
    for name, meta in layers.items():
        if meta.get("fingerprint") != fingerprints[name]:
            return False
        if meta["kind"] == "c12" and meta.get("base_mode") != base_mode:
            return False
    return True
