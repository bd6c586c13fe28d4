"""CPU checks of the C-ABI library: it loads, exports every symbol include/mbp.h declares, and rejects bad
arguments before touching the device.  No compute call runs here."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "mbp.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mbp_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("mbp_pack_c12", "mbp_pack_c12_escapes", "mbp_unpack_c12", "mbp_gemv_c12", "mbp_router_hilo",
              "mbp_status", "mbp_version"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    from mbp import _lib
    L = _lib.lib()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing


def test_binding_table_matches_header():
    from mbp import _lib
    assert sorted(n for n, _, _ in _lib.SIGNATURES) == declared_symbols()


def test_version_and_workspace_are_host_only():
    from mbp import _lib
    L = _lib.lib()
    assert L.mbp_version() == 1
    assert L.mbp_pack_c12_workspace(14336, 6144) == (14336 // 16) * 128 * 4
    assert L.mbp_pack_c12_workspace(15, 64) == 0  # bad shape


def test_argument_validation_without_device():
    from mbp import _lib
    L = _lib.lib()
    # null pointers are rejected before any CUDA call
    assert L.mbp_pack_c12(None, 64, 64, 1, None, None, None, None, 0, None) == -1
    assert L.mbp_gemv_c12(None, None, 1, 16, None, 16, None, None) == -1
    desc = _lib.C12(16, 16, 16, 0, 16, 64, 0)
    # n_out above the matrix height
    assert L.mbp_gemv_c12(ctypes.byref(desc), ctypes.c_void_p(16), 1, 32, ctypes.c_void_p(16), 32, None, None) == -2
    # misaligned x
    assert L.mbp_gemv_c12(ctypes.byref(desc), ctypes.c_void_p(18), 1, 16, ctypes.c_void_p(16), 16, None, None) == -4
    # token count
    assert L.mbp_gemv_c12(ctypes.byref(desc), ctypes.c_void_p(16), 0, 16, ctypes.c_void_p(16), 16, None, None) == -5
    # bad shapes for the packer
    assert L.mbp_pack_c12(ctypes.c_void_p(16), 20, 64, 1, ctypes.c_void_p(16), ctypes.c_void_p(16),
                          ctypes.c_void_p(16), ctypes.c_void_p(16), 4096, None) == -2
    assert L.mbp_pack_c12(ctypes.c_void_p(16), 16, 64, 7, ctypes.c_void_p(16), ctypes.c_void_p(16),
                          ctypes.c_void_p(16), ctypes.c_void_p(16), 4096, None) == -1


def test_device_check_without_gpu():
    import torch
    from mbp import _lib
    if torch.cuda.is_available():
        pytest.skip("device present")
    assert _lib.lib().mbp_device_check(0) == -10


def test_kernel_fn_rejects_bad_inputs():
    import torch
    import mbp
    state = {"layers": {}, "hilo": {}, "k": {}}
    with pytest.raises(ValueError):
        mbp.kernel_fn({"x": torch.zeros(2, 64), "config": {"m": 2, "n": 16, "k": 64, "layer": "o"}}, state)
    with pytest.raises(ValueError):
        mbp.kernel_fn({"x": torch.zeros(2, 64, dtype=torch.bfloat16), "config": {"m": 2, "n": 16, "k": 64,
                                                                                   "layer": "o"}}, state)
