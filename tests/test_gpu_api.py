"""The reference-facing API end to end on the GPU: prepare(weights) -> state, kernel_fn(data, state) -> out, with
the reference's own layer shapes (submission.py S:21-26) and its per-call contract (new output tensor each call,
unpooler n=1024 at M <= 8, FP32 router)."""
import pytest
import torch

from helpers import assert_close_bf16, assert_reference_norms, tokens, weight

pytestmark = pytest.mark.gpu

REF_SHAPES = {"qkv_gate": (2304, 8192), "o": (8192, 1024), "pooler": (4096, 8192), "unpooler": (8192, 4096)}


@pytest.fixture(scope="module")
def state_and_weights():
    import mbp
    ws = {name: weight(*shape, seed=i) for i, (name, shape) in enumerate(REF_SHAPES.items())}
    g = torch.Generator().manual_seed(9)
    ws["router"] = (torch.randn(256, 8192, generator=g) * 0.01).cuda()
    st = mbp.prepare(ws)
    return st, ws


@pytest.mark.parametrize("m", [1, 8, 16, 32, 128, 256])
@pytest.mark.parametrize("layer", ["qkv_gate", "o", "pooler", "unpooler", "router"])
def test_reference_shapes(state_and_weights, layer, m):
    import mbp
    st, ws = state_and_weights
    w = ws[layer]
    n = 1024 if layer == "unpooler" and m <= 8 else w.shape[0]
    x = tokens(m, w.shape[1], seed=m)
    data = {"x": x, "config": {"m": m, "n": n, "k": w.shape[1], "layer": layer}}
    out = mbp.kernel_fn(data, st)
    out2 = mbp.kernel_fn(data, st)
    assert out.data_ptr() != out2.data_ptr() and torch.equal(out, out2)
    assert out.shape == (m, n)
    if layer == "router":
        ref = x.double() @ w.double().T
        assert float((out.double() - ref).norm() / ref.norm()) <= 1e-5
    else:
        ref = x.float() @ w[:n].float().T
        assert_close_bf16(out, ref)
        assert_reference_norms(out, ref)
    assert mbp.device_status() == 0


def test_reference_spike_recipe(state_and_weights):
    """The reference's random-plus-spike input (S:305-310): the spike row is within 2.5e-4 (norm)."""
    import mbp
    st, ws = state_and_weights
    w = ws["o"]
    k = w.shape[1]
    gen = torch.Generator().manual_seed(11)
    for m in (1, 5, 8, 17, 32):
        x = torch.randn((m, k), generator=gen)
        x[m - 1].zero_()
        x[m - 1, (11 * 131 + m) % k] = 16.0
        x = x.to(torch.bfloat16).cuda()
        out = mbp.kernel_fn({"x": x, "config": {"m": m, "n": w.shape[0], "k": k, "layer": "o"}}, st)
        ref = (x.double() @ w.double().T).to(torch.bfloat16).double()
        d = (out.double() - ref)
        assert float(d[m - 1].norm() / ref[m - 1].norm()) <= 2.5e-4
        assert_reference_norms(out, ref)


def test_prepare_cache_round_trip(tmp_path, monkeypatch):
    """prepare(weights, cache=path): packs and writes on the first call, loads the same bytes on the next (no
    packing), and re-packs when a weight changes."""
    import mbp
    from mbp import ops
    ws = {"o": weight(1024, 512, seed=3, escape_frac=0.01), "router": (torch.randn(256, 512) * 0.01).cuda()}
    path = str(tmp_path / "w.mbp")
    st1 = mbp.prepare(ws, cache=path)
    packs = []
    real_c12, real_hilo = ops.pack_c12, ops.pack_hilo
    monkeypatch.setattr(mbp, "pack_c12", lambda *a, **k: packs.append(1) or real_c12(*a, **k))
    monkeypatch.setattr(mbp, "pack_hilo", lambda *a, **k: packs.append(1) or real_hilo(*a, **k))
    st2 = mbp.prepare(ws, cache=path)
    assert packs == []
    for name in ("units", "bases", "esc_off", "esc"):
        assert torch.equal(getattr(st1["layers"]["o"], name), getattr(st2["layers"]["o"], name))
    assert torch.equal(st1["hilo"]["router"].units, st2["hilo"]["router"].units)
    x = tokens(8, 512, seed=4)
    for layer, n in (("o", 1024), ("router", 256)):
        data = {"x": x, "config": {"m": 8, "n": n, "k": 512, "layer": layer}}
        assert torch.equal(mbp.kernel_fn(data, st1), mbp.kernel_fn(data, st2))
    ws2 = dict(ws, o=ws["o"].clone())
    ws2["o"][5, 7] = -ws2["o"][5, 7] + 1
    st3 = mbp.prepare(ws2, cache=path)
    assert len(packs) == 2  # every layer is packed again and the file rewritten
    data = {"x": x, "config": {"m": 8, "n": 1024, "k": 512, "layer": "o"}}
    assert_close_bf16(mbp.kernel_fn(data, st3), x.float() @ ws2["o"].float().T)
    assert mbp.device_status() == 0
