"""ctypes wrapper over the C port of the oracle (``c12_oracle.c``, built by ``oracle/Makefile``).

TEST INFRASTRUCTURE ONLY: used by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs as the
checker.  The numpy restatement in ``c12.py`` is the readable oracle; this module is its fast twin for
full-size matrices (up to 14336 x 6144), and ``tests/test_oracle_c.py`` checks that the two agree bit for bit.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE, "CC=gcc"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.orc_pack_c12.argtypes = [P, I, I, I, P, P, P, P, I64]
        L.orc_pack_c12.restype = I64
        L.orc_unpack_c12.argtypes = [P, P, P, P, I, I, P]
        L.orc_gemv_c12.argtypes = [P, I, P, P, P, P, I, I, I, I, P, P, I]
        L.orc_linear_f64.argtypes = [P, P, I, I, I, P, I]
        L.orc_linear_xbf16_wf32_f64.argtypes = [P, P, I, I, I, P, I]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def pack(w_bits: np.ndarray, tile_base: bool = True) -> dict:
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    n, k = w.shape
    r, c = n // 16, k // 64
    units = np.empty((r, c, 1536), dtype=np.uint8)
    bases = np.empty(r, dtype=np.uint8)
    off = np.empty(r * c + 1, dtype=np.int32)
    ne = lib().orc_pack_c12(_p(w), n, k, int(tile_base), _p(units), _p(bases), _p(off), None, 0)
    if ne < 0:
        raise ValueError(f"orc_pack_c12 failed: {ne}")
    esc = np.empty(max(int(ne), 1), dtype=np.uint32)
    ne2 = lib().orc_pack_c12(_p(w), n, k, int(tile_base), _p(units), _p(bases), _p(off), _p(esc), esc.size)
    assert ne2 == ne
    return {"n": n, "k": k, "units": units, "bases": bases, "esc_off": off, "esc": esc[:ne]}


def unpack(p: dict) -> np.ndarray:
    w = np.empty((p["n"], p["k"]), dtype=np.uint16)
    esc = p["esc"] if p["esc"].size else np.zeros(1, dtype=np.uint32)
    rc = lib().orc_unpack_c12(_p(p["units"]), _p(p["bases"]), _p(p["esc_off"]), _p(esc), p["n"], p["k"], _p(w))
    assert rc == 0
    return w


def gemv_packed(x_bits: np.ndarray, p: dict, row0: int = 0, nrows: int | None = None, threads: int = 0):
    """(out_f32 [m, n], out_bf16 [m, n]) from the packed format; rows outside [row0, row0+nrows) are zero."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    m = x.shape[0]
    n, k = p["n"], p["k"]
    nrows = n if nrows is None else nrows
    of = np.zeros((m, n), dtype=np.float32)
    ob = np.zeros((m, n), dtype=np.uint16)
    esc = p["esc"] if p["esc"].size else np.zeros(1, dtype=np.uint32)
    rc = lib().orc_gemv_c12(_p(x), m, _p(p["units"]), _p(p["bases"]), _p(p["esc_off"]), _p(esc), n, k, row0, nrows,
                            _p(of), _p(ob), threads)
    assert rc == 0
    return of, ob


def linear_f64(x_bits: np.ndarray, w_bits: np.ndarray, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    out = np.empty((x.shape[0], w.shape[0]), dtype=np.float64)
    lib().orc_linear_f64(_p(x), _p(w), x.shape[0], w.shape[0], x.shape[1], _p(out), threads)
    return out


def linear_wf32_f64(x_bits: np.ndarray, w_f32: np.ndarray, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w_f32, dtype=np.float32)
    out = np.empty((x.shape[0], w.shape[0]), dtype=np.float64)
    lib().orc_linear_xbf16_wf32_f64(_p(x), _p(w), x.shape[0], w.shape[0], x.shape[1], _p(out), threads)
    return out
