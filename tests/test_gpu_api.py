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
