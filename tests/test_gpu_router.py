"""FP32 router through the BF16 hi/lo pair: within 1e-5 (relative, norm) of an FP64 reference (BASELINE config
4), for M in {1, 8, 16, 32, 128, 256}, and one-hot exact against hi + lo (the reference's sm_exact, S:320-324)."""
import numpy as np
import pytest
import torch

from helpers import bits_np, tokens
from oracle import oracle

pytestmark = pytest.mark.gpu


def router_weight(n=256, k=6144, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * 0.01).cuda()


@pytest.mark.parametrize("m", [1, 8, 16, 32, 128, 256])
def test_router_vs_fp64(m):
    import mbp
    w = router_weight()
    p = mbp.pack_hilo(w)
    x = tokens(m, 6144, seed=m)
    out = mbp.router(p, x)
    ref = oracle.linear_wf32_f64(bits_np(x), w.cpu().numpy())
    got = out.double().cpu().numpy()
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel <= 1e-5, rel
    rows = np.linalg.norm(got - ref, axis=1) / np.linalg.norm(ref, axis=1)
    assert rows.max() <= 1e-5, rows.max()
    assert mbp.device_status() == 0


def test_router_onehot_equals_hi_plus_lo():
    import mbp
    w = router_weight(256, 1024, seed=3)
    p = mbp.pack_hilo(w)
    hi = w.to(torch.bfloat16)
    lo = (w - hi.float()).to(torch.bfloat16)
    exact = hi.float() + lo.float()
    for start in range(0, 1024, 32):
        x = torch.zeros(32, 1024, dtype=torch.bfloat16, device="cuda")
        x[torch.arange(32), torch.arange(start, start + 32)] = 1.0
        out = mbp.router(p, x)
        assert torch.equal(out, exact[:, start:start + 32].T.contiguous())


def test_router_through_api():
    import mbp
    w = router_weight()
    st = mbp.prepare({"router": w})
    x = tokens(8, 6144, seed=2)
    out = mbp.kernel_fn({"x": x, "config": {"m": 8, "n": 256, "k": 6144, "layer": "router"}}, st)
    assert out.dtype == torch.float32 and out.shape == (8, 256)
    ref = x.double() @ w.double().T
    assert float((out.double() - ref).norm() / ref.norm()) <= 1e-5
