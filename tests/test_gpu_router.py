"""FP32 router through the BF16 hi/lo pair: within 1e-5 (relative, norm) of an FP64 reference (6144 -> 256
experts), for M in {1, 8, 16, 32, 128, 256}, and one-hot exact against hi + lo (the reference's sm_exact, S:320-324).
The tensor-core path (M >= 64) is also checked at every token tile / cluster split it accepts, at the reference's
own 8192-column router, on ragged token counts and expert counts, one-hot exact, and for identical bits on repeats."""
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


def _rel_fp64(out, x, w):
    ref = oracle.linear_wf32_f64(bits_np(x), w.cpu().numpy())
    got = out.double().cpu().numpy()
    rows = np.linalg.norm(got - ref, axis=1) / np.linalg.norm(ref, axis=1)
    return np.linalg.norm(got - ref) / np.linalg.norm(ref), rows.max()


@pytest.mark.parametrize("m,k,n", [(64, 6144, 256), (100, 6144, 256), (128, 8192, 256), (256, 8192, 256),
                                   (300, 6144, 256), (70, 1024, 96), (512, 2048, 128)])
def test_router_tc_vs_fp64(m, k, n):
    import mbp
    w = router_weight(n, k, seed=m)
    p = mbp.pack_hilo(w)
    x = tokens(m, k, seed=m + 1)
    for out in (mbp.router_tc(p, x), mbp.router(p, x)):  # the tensor-core path and the default route
        rel, row = _rel_fp64(out, x, w)
        assert rel <= 1e-5 and row <= 1e-5, (rel, row)
    assert mbp.device_status() == 0


@pytest.mark.parametrize("bn,split", [(16, 3), (32, 8), (64, 16), (64, 4), (128, 3), (128, 16), (48, 12)])
def test_router_tc_geometries(bn, split):
    import mbp
    w = router_weight(256, 6144, seed=5)
    p = mbp.pack_hilo(w)
    x = tokens(256, 6144, seed=6)
    out = mbp.router_tc(p, x, bn=bn, split=split)
    rel, row = _rel_fp64(out, x, w)
    assert rel <= 1e-5 and row <= 1e-5, (bn, split, rel, row)
    again = mbp.router_tc(p, x, bn=bn, split=split)
    assert torch.equal(out, again)  # fixed reduction order: identical bits
    assert mbp.device_status() == 0


def test_router_tc_onehot_equals_hi_plus_lo():
    import mbp
    w = router_weight(256, 1024, seed=4)
    p = mbp.pack_hilo(w)
    hi = w.to(torch.bfloat16)
    lo = (w - hi.float()).to(torch.bfloat16)
    exact = hi.float() + lo.float()
    for start in range(0, 1024, 128):
        x = torch.zeros(128, 1024, dtype=torch.bfloat16, device="cuda")
        x[torch.arange(128), torch.arange(start, start + 128)] = 1.0
        out = mbp.router_tc(p, x, split=4)
        assert torch.equal(out, exact[:, start:start + 128].T.contiguous()), start


def test_router_tc_rejects_bad_geometry():
    import mbp
    p = mbp.pack_hilo(router_weight(256, 1024))
    x = tokens(64, 1024)
    for bn, split in ((24, 0), (256, 0), (0, 17), (0, 32)):
        with pytest.raises(mbp.MbpError):
            mbp.router_tc(p, x, bn=bn, split=split)
    # a cluster too small for the accuracy bound: at most 2048 columns per CTA (6144 -> split >= 3)
    p = mbp.pack_hilo(router_weight(256, 6144))
    x = tokens(64, 6144)
    for bn, split in ((16, 1), (64, 2)):
        with pytest.raises(mbp.MbpError):
            mbp.router_tc(p, x, bn=bn, split=split)


def test_router_through_api():
    import mbp
    w = router_weight()
    st = mbp.prepare({"router": w})
    x = tokens(8, 6144, seed=2)
    out = mbp.kernel_fn({"x": x, "config": {"m": 8, "n": 256, "k": 6144, "layer": "router"}}, st)
    assert out.dtype == torch.float32 and out.shape == (8, 256)
    ref = x.double() @ w.double().T
    assert float((out.double() - ref).norm() / ref.norm()) <= 1e-5


def _topk_reference(logits: torch.Tensor, k: int, renorm: bool):
    """Row-wise: ids by (value descending, index ascending), NaN below every number; softmax in float64."""
    lg = logits.double().cpu()
    key = torch.where(torch.isnan(lg), torch.full_like(lg, float("-inf")), lg)
    ids, ws = [], []
    for row in key:
        order = sorted(range(row.numel()), key=lambda c: (-float(row[c]), c))[:k]
        sel = row[order]
        top = float(sel[0])
        ex = torch.exp(sel - top)
        den = ex.sum() if renorm else torch.exp(row - top).sum()
        ids.append(order)
        ws.append((ex / den).tolist())
    return torch.tensor(ws, dtype=torch.float64), torch.tensor(ids, dtype=torch.int32)


@pytest.mark.parametrize("m,e,k", [(1, 256, 8), (8, 256, 1), (33, 256, 2), (256, 256, 8), (5, 100, 32),
                                   (3, 1024, 4), (17, 64, 64 // 2)])
@pytest.mark.parametrize("renorm", [True, False])
def test_router_topk(m, e, k, renorm):
    import mbp
    g = torch.Generator().manual_seed(m * 1000 + e + k)
    logits = torch.randn(m, e, generator=g) * 3
    logits[0, : e // 4] = torch.round(logits[0, : e // 4])  # ties: lower index first
    if m > 2:
        logits[2, 5] = float("nan")
    w, ids = mbp.router_topk(logits.cuda(), k, renorm)
    rw, rids = _topk_reference(logits, k, renorm)
    assert torch.equal(ids.cpu(), rids)
    assert torch.allclose(w.cpu().double(), rw, rtol=1e-5, atol=1e-7)
    assert mbp.device_status() == 0


def test_route_on_prepared_router():
    import mbp
    g = torch.Generator().manual_seed(21)
    wr = (torch.randn(256, 6144, generator=g) * 0.01).cuda()
    st = mbp.prepare({"router": wr})
    x = (torch.randn(32, 6144, generator=g)).to(torch.bfloat16).cuda()
    data = {"x": x, "config": {"m": 32, "n": 256, "k": 6144, "layer": "router"}}
    w, ids = mbp.route(data, st, 8)
    w2, ids2 = mbp.router_topk(mbp.kernel_fn(data, st), 8)
    assert torch.equal(ids, ids2) and torch.equal(w, w2)
    assert torch.allclose(w.sum(1), torch.ones(32, device="cuda"), atol=1e-6)
