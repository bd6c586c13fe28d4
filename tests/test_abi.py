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


def test_ctypes_structs_mirror_the_header(tmp_path):
    """Sizes and field offsets of the ctypes mirrors equal the C structs of include/mbp.h (compiled by gcc)."""
    import shutil
    import subprocess
    from mbp import _lib
    gcc = shutil.which("gcc")
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    if gcc is None or not os.path.exists(os.path.join(cuda_inc, "cuda_runtime.h")):
        pytest.skip("gcc or the CUDA headers are missing")
    mirrors = {"mbp_c12": _lib.C12, "mbp_hilo": _lib.HiLo, "mbp_gemv_geom": _lib.Geom,
               "mbp_tp_exchange": _lib.TPExchange}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "mbp.h"', "int main(void) {"]
    for cname, py in mirrors.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([gcc, str(src), "-I", os.path.join(ROOT, "include"), "-I", cuda_inc, "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        parts = line.split()
        got[(parts[0], parts[1])] = int(parts[2])
    for cname, py in mirrors.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


def test_exchange_entry_points_validate_without_device():
    from mbp import _lib
    L = _lib.lib()
    desc = _lib.C12(16, 16, 16, 0, 32, 64, 0)
    ex = _lib.TPExchange()
    ex.bufs[0], ex.bufs[1] = 4096, 8192
    ex.parity_stride, ex.counter, ex.rank, ex.P, ex.mode, ex.n = 1024, 64, 0, 2, _lib.TP_GATHER_BF16, 64
    call = lambda d, e, m=1, out=16: L.mbp_gemv_c12_tp(ctypes.byref(d), ctypes.c_void_p(16), 64, m, ctypes.byref(e),
                                                        ctypes.c_void_p(out), None, None)
    assert L.mbp_gemv_c12_tp(None, None, 64, 1, None, None, None, None) == -1
    ex.P = 9
    assert call(desc, ex) == -2                      # rank count above 8
    ex.P, ex.mode = 2, 7
    assert call(desc, ex) == -1                      # unknown exchange mode
    ex.mode, ex.n = _lib.TP_GATHER_BF16, 48
    assert call(desc, ex) == -2                      # gathered width != P * shard rows
    ex.n = 64
    assert call(desc, ex, m=33) == -5                # the fused exchange is the GEMV's (m <= 32)
    assert call(desc, ex, out=24) == -4              # misaligned output
    ex.counter = None
    assert call(desc, ex) == -1
    # the receive kernel: bad rank / mode before any launch
    flags = (ctypes.c_void_p * 2)(16, 32)
    assert L.mbp_tp_finish(flags, 2, 2, ctypes.c_void_p(64), None, 0, _lib.TP_BARRIER, 0, 0, None, None) == -2
    assert L.mbp_tp_finish(flags, 0, 2, ctypes.c_void_p(64), None, 0, 9, 1, 16, None, None) == -1
    assert L.mbp_tp_finish(flags, 0, 2, ctypes.c_void_p(64), ctypes.c_void_p(16), 0, _lib.TP_GATHER_BF16, 1, 20,
                           ctypes.c_void_p(16), None) == -2


def test_router_topk_validates_without_device():
    from mbp import _lib
    L = _lib.lib()
    p = ctypes.c_void_p(16)
    assert L.mbp_router_topk(None, 1, 256, 256, 8, 1, p, p, None) == -1
    assert L.mbp_router_topk(p, 0, 256, 256, 8, 1, p, p, None) == -5
    assert L.mbp_router_topk(p, 1, 256, 256, 33, 1, p, p, None) == -2   # k above 32
    assert L.mbp_router_topk(p, 1, 4, 4, 8, 1, p, p, None) == -2        # k above e
    assert L.mbp_router_topk(p, 1, 2048, 2048, 8, 1, p, p, None) == -2  # e above 1024
    assert L.mbp_router_topk(p, 1, 256, 128, 8, 1, p, p, None) == -2    # row stride below e
    assert L.mbp_router_topk(p, 1, 256, 256, 8, 2, p, p, None) == -1    # renorm flag
    assert L.mbp_router_topk(ctypes.c_void_p(18), 1, 256, 256, 8, 1, p, p, None) == -4
