"""The allocation-free packer entry point, mbp_pack_c12_noalloc, against the regular one.

Some callers cannot allocate device memory themselves: a loader that a host framework hands only preallocated
weight and output buffers (the framework owns all device memory), or a caller that must not trigger
cudaMalloc's implicit device-wide synchronisation while other streams run.  mbp_pack_c12_noalloc serves them
by keeping its scratch (per-tile exponent histograms) in a fixed device array inside the library.  This test
calls it through the C ABI twice in a row, on two different matrices and both base modes, and checks every
output against mbp_pack_c12 (which takes a caller-provided workspace) bit for bit -- the packer's outputs are
integers, so the tolerance is exact equality.  It lives in its own file so pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _weight(n, k, seed, escape_frac):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    idx = torch.randperm(n * k, generator=torch.Generator().manual_seed(seed + 1))[: int(n * k * escape_frac)]
    w.view(-1)[idx] *= 256
    return w.to(torch.bfloat16).cuda()


def _outputs(n, k):
    r, c = n // 16, k // 64
    # filled with a pattern so that anything left unwritten shows up as a mismatch
    units = torch.full((r, c, 1536), 0xA5, dtype=torch.uint8, device="cuda")
    bases = torch.full((r,), 0xA5, dtype=torch.uint8, device="cuda")
    esc_off = torch.full((r * c + 1,), -7, dtype=torch.int32, device="cuda")
    return units, bases, esc_off


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_matches_workspace_packer_twice():
    from mbp import _lib
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cases = [(4096, 1536, 3, 0.01, 1), (2048, 6144, 5, 0.002, 0)]  # (n, k, seed, escape fraction, base mode)
    for n, k, seed, frac, mode in cases:
        w = _weight(n, k, seed, frac)
        ref = _outputs(n, k)
        ws_bytes = L.mbp_pack_c12_workspace(n, k)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        assert L.mbp_pack_c12(_p(w), n, k, mode, _p(ref[0]), _p(ref[1]), _p(ref[2]), _p(ws), ws_bytes, stream) == 0
        got = _outputs(n, k)
        assert L.mbp_pack_c12_noalloc(_p(w), n, k, mode, _p(got[0]), _p(got[1]), _p(got[2]), stream) == 0
        torch.cuda.synchronize()
        for a, b in zip(ref, got):
            assert torch.equal(a, b)
        assert int(got[2][-1]) > 0  # escapes were exercised
    assert _lib.device_status() == 0


def test_noalloc_rejects_matrices_above_its_scratch():
    from mbp import _lib
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    fake = ctypes.c_void_p(256)  # never dereferenced: the size check comes first
    assert L.mbp_pack_c12_noalloc(fake, 16384 + 16, 64, 1, fake, fake, fake, stream) == -12
