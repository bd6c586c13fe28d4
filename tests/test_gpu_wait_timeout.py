"""Bounded device waits give up with a status instead of hanging or trapping.

Every wait in the library's kernels (pipeline stages, tensor-core completion, a peer's exchange words or barrier
flags) is bounded; when the limit runs out the kernel records an MBP_DEV_TIMEOUT_* code in the device status word
and returns, so the context stays usable (the reference traps after a 20 ms spin instead, submission.py
S:46<105-111>).  These tests make a peer wait run out on ONE GPU, without any fault: a tensor-parallel exchange
of two ranks in which the "other rank" is a zeroed buffer that nothing ever writes.  The wait limit is lowered
to 2 ms for them (mbp_set_wait_limit), so each call returns within milliseconds; the status word must then read
MBP_DEV_TIMEOUT_PEER, reading it with clear must reset it, and the device must still run a normal GEMV exactly.
"""
import ctypes
import time

import pytest
import torch

from helpers import assert_close_bf16, tokens, weight

pytestmark = pytest.mark.gpu

TIMEOUT_PEER = 4  # MBP_DEV_TIMEOUT_PEER
LIMIT_NS = 2_000_000


@pytest.fixture
def short_waits():
    import mbp
    assert mbp.device_status() == 0
    prev = mbp.set_wait_limit(LIMIT_NS)
    try:
        yield
    finally:
        torch.cuda.synchronize()
        mbp.set_wait_limit(0)
    assert prev == 1_000_000_000  # the default limit was in force before


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _timed(fn):
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    return time.perf_counter() - t0


def _still_exact():
    """After a timed-out wait the context is intact: a plain GEMV matches the FP32 reference."""
    import mbp
    w = weight(256, 512, seed=3)
    x = tokens(8, 512, seed=4)
    assert_close_bf16(mbp.gemv(mbp.pack_c12(w), x), x.float() @ w.float().T)
    assert mbp.device_status() == 0


def test_flag_barrier_times_out(short_waits):
    import mbp
    from mbp._lib import TP_BARRIER, check, lib
    own = torch.zeros(8, dtype=torch.int32, device="cuda")
    peer = torch.zeros(8, dtype=torch.int32, device="cuda")  # rank 1's flag array: nobody announces into it
    counter = torch.zeros(65, dtype=torch.int32, device="cuda")
    flags = (ctypes.c_void_p * 2)(own.data_ptr(), peer.data_ptr())
    dt = _timed(lambda: check(lib().mbp_tp_finish(flags, 0, 2, ctypes.c_void_p(counter.data_ptr()), None, 0,
                                                  TP_BARRIER, 0, 0, None, _stream()), "mbp_tp_finish"))
    assert dt < 1.0
    assert int(peer[0]) == 1 and int(own[0]) == 1  # this rank announced epoch 1 to both arrays
    assert mbp.device_status() == TIMEOUT_PEER     # ... and gave up waiting for rank 1's announcement
    assert mbp.device_status() == 0                # reading with clear reset the word
    _still_exact()


@pytest.mark.parametrize("mode", ["gather", "sum"])
def test_receive_kernel_times_out(short_waits, mode):
    """The two-kernel form's receive step waits for words tagged with the new epoch; none ever arrive."""
    import mbp
    from mbp._lib import TP_GATHER_BF16, TP_SUM_F32, check, lib
    m, n, P = 4, 256, 2
    words = m * n // 2 if mode == "gather" else P * m * n
    buf = torch.zeros(2 * words, dtype=torch.int64, device="cuda")
    counter = torch.zeros(65, dtype=torch.int32, device="cuda")
    out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    code = TP_GATHER_BF16 if mode == "gather" else TP_SUM_F32
    dt = _timed(lambda: check(lib().mbp_tp_finish(None, 0, P, ctypes.c_void_p(counter.data_ptr()),
                                                  ctypes.c_void_p(buf.data_ptr()), words * 8, code, m, n,
                                                  ctypes.c_void_p(out.data_ptr()), _stream()), "mbp_tp_finish"))
    assert dt < 1.0
    assert mbp.device_status() == TIMEOUT_PEER
    assert mbp.device_status() == 0
    assert bool((counter[:64] == 1).all())  # the epoch still advanced: the next exchange stays in step
    _still_exact()


@pytest.mark.parametrize("mode", ["gather", "sum"])
def test_fused_exchange_times_out(short_waits, mode):
    """The one-kernel form (mbp_gemv_c12_tp): the GEMV stores its words into both ranks' buffers (the second is
    a local stand-in), then each CTA waits for rank 1's words in its own buffer, which nobody writes."""
    import mbp
    from mbp._lib import TP_GATHER_BF16, TP_SUM_F32, TPExchange, check, lib
    m, P = 8, 2
    ns, k = 512, 1024
    w = weight(ns, k, seed=5)
    p = mbp.pack_c12(w)
    x = tokens(m, k * (P if mode == "sum" else 1), seed=6)
    n = ns * P if mode == "gather" else ns
    words = 32 * n // 2 if mode == "gather" else P * 32 * n
    bufs = [torch.zeros(2 * words, dtype=torch.int64, device="cuda") for _ in range(P)]
    counter = torch.zeros(65, dtype=torch.int32, device="cuda")
    out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    ex = TPExchange()
    for r in range(P):
        ex.bufs[r] = bufs[r].data_ptr()
    ex.parity_stride = words * 8
    ex.counter = counter.data_ptr()
    ex.rank, ex.P, ex.n = 0, P, n
    ex.mode = TP_GATHER_BF16 if mode == "gather" else TP_SUM_F32
    dt = _timed(lambda: check(lib().mbp_gemv_c12_tp(ctypes.byref(p.desc), ctypes.c_void_p(x.data_ptr()), x.shape[1],
                                                    m, ctypes.byref(ex), ctypes.c_void_p(out.data_ptr()), None,
                                                    _stream()), "mbp_gemv_c12_tp"))
    assert dt < 1.0
    assert mbp.device_status() == TIMEOUT_PEER
    assert mbp.device_status() == 0
    # this rank's own words did arrive in the stand-in peer buffer, tagged with epoch 1
    assert bool(((bufs[1].view(-1) >> 32) == 1).any())
    _still_exact()
