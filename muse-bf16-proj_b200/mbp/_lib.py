"""ctypes binding of libmbp.so (the C ABI declared in include/mbp.h).

The product path has no CPU fallback: if the library is missing or the device is not an sm_100 part, every
call raises.  Build the library with ``python muse-bf16-proj_b200/build.py``.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmbp.so")

STATUS_NAMES = {
    -1: "bad argument", -2: "bad shape", -3: "impossible geometry", -4: "pointer not 16-byte aligned",
    -5: "token count out of range", -6: "shared memory above device limit", -8: "kernel launch failed",
    -9: "cluster shape not schedulable", -10: "device is not sm_100", -11: "buffer too small",
    -12: "matrix too tall for the allocation-free packer's fixed scratch (n > 16384)",
    -100: "tensor-map encode failed",
}

DEVICE_STATUS = {1: "consumer timed out waiting for a stage", 2: "producer timed out waiting for a stage to drain",
                 3: "tensor-core completion timed out", 4: "a peer rank's barrier flag did not arrive"}


TP_COUNTER_SLOTS = 64                                    # MBP_TP_COUNTER_SLOTS
TP_BARRIER, TP_GATHER_BF16, TP_SUM_F32 = 0, 1, 2         # MBP_TP_* modes of mbp_tp_finish
TP_RSAG = 3                                                # MBP_TP_RSAG: fused row-parallel reduce-scatter + gather
OUT_BF16, OUT_F32, OUT_TAGGED_BF16X2, OUT_TAGGED_F32 = 0, 1, 2, 3  # MBP_OUT_* kinds of mbp_gemv_c12_multi


class MbpError(RuntimeError):
    def __init__(self, rc: int, what: str):
        super().__init__(f"{what}: status {rc} ({STATUS_NAMES.get(rc, 'unknown')})")
        self.rc = rc


class C12(ctypes.Structure):
    _fields_ = [("units", ctypes.c_void_p), ("bases", ctypes.c_void_p), ("esc_off", ctypes.c_void_p),
                ("esc", ctypes.c_void_p), ("n", ctypes.c_int32), ("k", ctypes.c_int32), ("n_esc", ctypes.c_int64)]


class HiLo(ctypes.Structure):
    _fields_ = [("units", ctypes.c_void_p), ("n", ctypes.c_int32), ("k", ctypes.c_int32)]


class TPExchange(ctypes.Structure):  # mirrors mbp_tp_exchange
    _fields_ = [("bufs", ctypes.c_void_p * 8), ("parity_stride", ctypes.c_longlong), ("counter", ctypes.c_void_p),
                ("rank", ctypes.c_int), ("P", ctypes.c_int), ("mode", ctypes.c_int), ("n", ctypes.c_int)]


class Geom(ctypes.Structure):
    _fields_ = [("rb", ctypes.c_int32), ("rtw", ctypes.c_int32), ("split", ctypes.c_int32),
                ("wki", ctypes.c_int32), ("kci", ctypes.c_int32), ("stages", ctypes.c_int32),
                ("nblk", ctypes.c_int32)]

    def as_tuple(self):
        return (self.rb, self.rtw, self.split, self.wki, self.kci, self.stages, self.nblk)


# (name, restype, argtypes) for every symbol of include/mbp.h
_P, _I, _I64, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = [
    ("mbp_version", _I, []),
    ("mbp_device_check", _I, [_I]),
    ("mbp_status", _I, [ctypes.POINTER(ctypes.c_int), _I]),
    ("mbp_set_wait_limit", ctypes.c_ulonglong, [ctypes.c_ulonglong]),
    ("mbp_pack_c12_workspace", _SZ, [_I, _I]),
    ("mbp_pack_c12", _I, [_P, _I, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    ("mbp_pack_c12_noalloc", _I, [_P, _I, _I, _I, _P, _P, _P, _P]),
    ("mbp_pack_c12_escapes", _I, [_P, _I, _I, _P, _P, _P, _P]),
    ("mbp_unpack_c12", _I, [ctypes.POINTER(C12), _P, _P]),
    ("mbp_pack_hilo", _I, [_P, _I, _I, _P, _P]),
    ("mbp_gemv_plan", _I, [_I, _I, _I, ctypes.POINTER(Geom)]),
    ("mbp_gemv_plan_ex", _I, [_I, _I, _I, _I, ctypes.POINTER(Geom)]),
    ("mbp_gemv_c12", _I, [ctypes.POINTER(C12), _P, _I, _I, _P, _I, ctypes.POINTER(Geom), _P]),
    ("mbp_gemv_c12_f32", _I, [ctypes.POINTER(C12), _P, _I, _I, _P, _I, ctypes.POINTER(Geom), _P]),
    ("mbp_router_hilo", _I, [ctypes.POINTER(HiLo), _P, _I, _P, _I, ctypes.POINTER(Geom), _P]),
    ("mbp_router_topk", _I, [_P, _I, _I, _I, _I, _I, _P, _P, _P]),
    ("mbp_tp_assemble_columns", _I, [_P, _P, _I, _I, _I, _P]),
    ("mbp_f32_to_bf16", _I, [_P, _P, ctypes.c_longlong, _P]),
    ("mbp_ipc_alloc", _I, [_SZ, ctypes.POINTER(ctypes.c_void_p), _P]),
    ("mbp_ipc_open", _I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    ("mbp_ipc_close", _I, [_P]),
    ("mbp_ipc_free", _I, [_P]),
    ("mbp_gemv_c12_multi", _I, [ctypes.POINTER(C12), _P, _I, _I, _I, ctypes.POINTER(ctypes.c_void_p), _I, _I, _I,
                                _P, ctypes.c_longlong, ctypes.POINTER(Geom), _P]),
    ("mbp_tp_finish", _I, [ctypes.POINTER(ctypes.c_void_p), _I, _I, _P, _P, ctypes.c_longlong, _I, _I, _I, _P,
                           _P]),
    ("mbp_gemv_c12_tp", _I, [ctypes.POINTER(C12), _P, _I, _I, ctypes.POINTER(TPExchange), _P, ctypes.POINTER(Geom),
                             _P]),
    ("mbp_gemm_c12", _I, [ctypes.POINTER(C12), _P, _I, _I, _P, _I, _P]),
    ("mbp_gemm_c12_f32", _I, [ctypes.POINTER(C12), _P, _I, _I, _P, _I, _P]),
    ("mbp_router_hilo_tc", _I, [ctypes.POINTER(HiLo), _P, _I, _P, _I, _I, _I, _P]),
    ("mbp_gemm_c12_multi", _I, [ctypes.POINTER(C12), _P, _I, _I, ctypes.POINTER(_P), _I, _I, _I, _P, _I64, _P]),
]

_lib = None
_lock = threading.Lock()


def lib():
    """Loads libmbp.so once; raises when it is missing (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python muse-bf16-proj_b200/build.py`")
            L = ctypes.CDLL(LIB_PATH)
            for name, res, args in SIGNATURES:
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise MbpError(rc, what)


def set_wait_limit(ns: int) -> int:
    """Limit (ns) of every bounded device wait in kernels launched from now on (0: the default 1 s); returns the
    previous one.  A wait that runs out sets its MBP_DEV_TIMEOUT_* code in the status word (``device_status``)."""
    return int(lib().mbp_set_wait_limit(int(ns)))


def device_status(clear: bool = True) -> int:
    v = ctypes.c_int(0)
    check(lib().mbp_status(ctypes.byref(v), int(clear)), "mbp_status")
    return v.value
