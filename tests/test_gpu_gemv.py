"""GEMV parity on the GPU through the C ABI.

* one-hot exactness (the reference's sm_verify_onehot, S:281-294): x = e_k rows must reproduce W[:, k] bit for
  bit, which pins decode, escape patching, fragment mapping and output indexing;
* random inputs against the oracle (C port, sampled rows) and an FP32 reference, tolerance
  rtol 1e-2 / atol 1e-2, plus the reference's own norm rule (S:297-317);
* the decode shapes (QKV+gate 6144->14336, O 6144->6144) at M in {1, 8, 16, 32} with and without the 1% x256
  escape variant, every token count 1..33 on a small matrix, M > 32 (token blocks), n_out < n (the reference's unpooler n=1024), FP32 output.
"""
import numpy as np
import pytest
import torch

from helpers import assert_close_bf16, assert_reference_norms, bits_np, tokens, weight
from oracle import oracle

pytestmark = pytest.mark.gpu


def ref_f32(x, w, n_out=None):
    n_out = w.shape[0] if n_out is None else n_out
    return x.float() @ w[:n_out].float().T


def onehot_check(p, w, cols, n_out=None):
    import mbp
    n_out = w.shape[0] if n_out is None else n_out
    k = w.shape[1]
    for m in (1, 8, 32):
        for i in range(0, len(cols), m):
            cs = cols[i:i + m]
            x = torch.zeros(len(cs), k, dtype=torch.bfloat16, device="cuda")
            x[torch.arange(len(cs)), torch.tensor(cs, device="cuda")] = 1.0
            out = mbp.gemv(p, x, n_out=n_out)
            want = w[:n_out, cs].T
            assert torch.equal(out.view(torch.int16), want.contiguous().view(torch.int16)), (m, cs[:4])


@pytest.mark.parametrize("frac", [0.0, 0.01])
def test_onehot_exact_small(frac):
    import mbp
    w = weight(256, 1024, seed=3, escape_frac=frac)
    for mode in (mbp.BASE_MATRIX, mbp.BASE_TILE):
        p = mbp.pack_c12(w, mode)
        onehot_check(p, w, list(range(1024)))
    assert mbp.device_status() == 0


@pytest.mark.parametrize("shape", [(14336, 6144), (6144, 6144)])
@pytest.mark.parametrize("frac", [0.0, 0.01])
def test_onehot_exact_baseline_shapes(shape, frac):
    import mbp
    w = weight(*shape, seed=0, escape_frac=frac)
    p = mbp.pack_c12(w)
    g = torch.Generator().manual_seed(5)
    cols = torch.randperm(shape[1], generator=g)[:96].tolist() + [0, shape[1] - 1]
    onehot_check(p, w, cols)
    assert mbp.device_status() == 0


@pytest.mark.parametrize("m", list(range(1, 34)))
def test_every_token_count_small(m):
    import mbp
    w = weight(512, 768, seed=7, escape_frac=0.005)
    p = mbp.pack_c12(w)
    x = tokens(m, 768, seed=m)
    out = mbp.gemv(p, x)
    assert_close_bf16(out, ref_f32(x, w))


@pytest.mark.parametrize("shape", [(14336, 6144), (6144, 6144)])
@pytest.mark.parametrize("m", [1, 8, 16, 32])
@pytest.mark.parametrize("frac", [0.0, 0.01])
def test_baseline_config2(shape, m, frac):
    """The decode shapes against the FP32 reference and, over the whole output, the C oracle (which decodes the
    packed bytes on the host and accumulates in FP32); both the GEMV and the public kernel_fn route."""
    import mbp
    w = weight(*shape, seed=0, escape_frac=frac)
    st = mbp.prepare({"o": w})
    p = st["layers"]["o"]
    x = tokens(m, shape[1], seed=1)
    out = mbp.gemv(p, x)
    api = mbp.kernel_fn({"x": x, "config": {"m": m, "n": shape[0], "k": shape[1], "layer": "o"}}, st)
    torch.cuda.synchronize()
    assert mbp.device_status() == 0
    ref = ref_f32(x, w)
    for o in (out, api):
        assert_close_bf16(o, ref)
        assert_reference_norms(o, ref)
    host = {"n": p.n, "k": p.k, "units": p.units.cpu().numpy(), "bases": p.bases.cpu().numpy(),
            "esc_off": p.esc_off.cpu().numpy(), "esc": p.esc.cpu().numpy().view(np.uint32)}
    of, ob = oracle.gemv_packed(bits_np(x), host)
    for o in (out, api):
        assert np.allclose(o.float().cpu().numpy(), of, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("m", [33, 64, 128, 256])
def test_token_blocks_beyond_32(m):
    import mbp
    w = weight(1536, 6144, seed=2)
    p = mbp.pack_c12(w)
    x = tokens(m, 6144, seed=4)
    out = mbp.gemv(p, x)
    assert_close_bf16(out, ref_f32(x, w))


def test_partial_rows_unpooler_style():
    """The reference's unpooler at M <= 8 computes only the first 1024 rows (S:272-273)."""
    import mbp
    w = weight(8192, 4096, seed=9)
    p = mbp.pack_c12(w)
    for m in (1, 8):
        x = tokens(m, 4096, seed=m)
        out = mbp.gemv(p, x, n_out=1024)
        assert out.shape == (m, 1024)
        assert_close_bf16(out, ref_f32(x, w, 1024))


def test_f32_output_and_strided_out():
    import mbp
    w = weight(6144, 1536, seed=11)
    p = mbp.pack_c12(w)
    x = tokens(5, 1536, seed=3)
    big = torch.full((5, 7000), float("nan"), device="cuda")
    out = mbp.gemv(p, x, out=big)
    ref = ref_f32(x, w)
    assert torch.allclose(out[:, :6144], ref, rtol=1e-5, atol=1e-4)
    assert bool(torch.isnan(big[:, 6144:]).all())


def test_explicit_geometries_agree():
    """Several launch geometries (split-K by cluster, warp K split, stage depth) give the same result."""
    import mbp
    from mbp._lib import Geom
    w = weight(1024, 3072, seed=12, escape_frac=0.01)
    p = mbp.pack_c12(w)
    x = tokens(8, 3072, seed=1)
    ref = mbp.gemv(p, x, out_dtype=torch.float32)
    for g in [Geom(8, 1, 1, 1, 4, 2), Geom(4, 1, 3, 2, 4, 3), Geom(2, 1, 8, 4, 4, 2), Geom(1, 1, 6, 3, 4, 2),
              Geom(11, 1, 2, 1, 4, 2), Geom(3, 1, 1, 2, 8, 2), Geom(3, 1, 1, 2, 4, 2, 23),
              Geom(8, 1, 2, 1, 4, 2, 9)]:
        out = mbp.gemv(p, x, out_dtype=torch.float32, geom=g)
        # same FP32 products, different split-K summation order
        assert torch.allclose(out, ref, rtol=1e-4, atol=1e-3), g.as_tuple()
    assert mbp.device_status() == 0


def test_zero_and_tiny_matrices():
    import mbp
    for n, k in [(16, 64), (32, 128), (48, 64)]:
        w = weight(n, k, seed=n + k)
        p = mbp.pack_c12(w)
        x = tokens(3, k)
        assert_close_bf16(mbp.gemv(p, x), ref_f32(x, w))
    w = torch.zeros(64, 256, dtype=torch.bfloat16, device="cuda")
    p = mbp.pack_c12(w)
    assert bool((mbp.gemv(p, tokens(4, 256)) == 0).all())
