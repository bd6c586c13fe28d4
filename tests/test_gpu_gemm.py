"""tcgen05 verify GEMM parity on the GPU through the C ABI.

* one-hot exactness (the reference's sm_verify_onehot idea, S:281-294): rows of x = e_k reproduce W[:, k] bit
  for bit, which pins the decode into shared memory, the swizzled operand layout, the UMMA descriptors and the
  TMEM epilogue mapping;
* the prefill shapes (M in {128, 256}; QKV+gate, O, pooler 6144->1536, unpooler 1536->6144) against the
  FP32 reference at rtol 1e-2 / atol 1e-2 plus the reference's norm rule (S:297-317);
* ragged token counts (tiles of up to 256 tokens, token tails), n_out < n, escape-heavy weights, FP32 output.
"""
import pytest
import torch

from helpers import assert_close_bf16, assert_reference_norms, tokens, weight

pytestmark = pytest.mark.gpu

CONFIG3 = {"qkv_gate": (14336, 6144), "o": (6144, 6144), "pooler": (1536, 6144), "unpooler": (6144, 1536)}


def ref_f32(x, w, n_out=None):
    n_out = w.shape[0] if n_out is None else n_out
    return x.float() @ w[:n_out].float().T


def test_gemm_onehot_exact():
    import mbp
    w = weight(384, 1024, seed=21, escape_frac=0.01)
    p = mbp.pack_c12(w)
    for start in range(0, 1024, 256):
        x = torch.zeros(256, 1024, dtype=torch.bfloat16, device="cuda")
        x[torch.arange(256), torch.arange(start, start + 256)] = 1.0
        out = mbp.gemm(p, x)
        assert torch.equal(out.view(torch.int16), w[:, start:start + 256].T.contiguous().view(torch.int16)), start
    assert mbp.device_status() == 0


@pytest.mark.parametrize("variant", ["plain", "esc1pct"])
@pytest.mark.parametrize("layer", list(CONFIG3))
@pytest.mark.parametrize("m", [128, 256])
def test_gemm_baseline_config3(layer, m, variant):
    import mbp
    n, k = CONFIG3[layer]
    w = weight(n, k, seed=0, escape_frac=0.01 if variant == "esc1pct" else 0.0)
    p = mbp.pack_c12(w)
    x = tokens(m, k, seed=m)
    out = mbp.gemm(p, x)
    torch.cuda.synchronize()
    assert mbp.device_status() == 0
    ref = ref_f32(x, w)
    assert_close_bf16(out, ref)
    assert_reference_norms(out, ref)


@pytest.mark.parametrize("m", [1, 17, 33, 48, 100, 200, 255, 257, 300, 512])
def test_gemm_token_counts(m):
    import mbp
    w = weight(1024, 2048, seed=m, escape_frac=0.005)
    p = mbp.pack_c12(w)
    x = tokens(m, 2048, seed=m + 1)
    out = mbp.gemm(p, x)
    assert_close_bf16(out, ref_f32(x, w))


@pytest.mark.parametrize("n,k,m", [(256, 64, 128), (256, 192, 64), (512, 320, 256), (1024, 7 * 64 * 9, 96),
                                   (768, 64 * 37, 200)])
def test_gemm_odd_chunk_counts(n, k, m):
    """K ranges with an odd number of 64-column chunks (a last stage holding one chunk), down to a single chunk,
    with and without a K split, on escape-bearing weights: within rtol 1e-4 / atol 1e-3 of the GEMV's FP32 output
    (the same products summed in another order) and within the BF16 tolerance of the FP32 reference."""
    import mbp
    w = weight(n, k, seed=k, escape_frac=0.01)
    p = mbp.pack_c12(w)
    x = tokens(m, k, seed=m)
    out = mbp.gemm(p, x, out_dtype=torch.float32)
    ref = torch.cat([mbp.gemv(p, x[i:i + 32].contiguous(), out_dtype=torch.float32) for i in range(0, m, 32)])
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-3)
    assert_close_bf16(mbp.gemm(p, x), ref_f32(x, w))
    assert mbp.device_status() == 0


@pytest.mark.parametrize("n,k,m", [(14288, 1024, 128), (14336, 576, 64), (12048, 640, 100)])
def test_gemm_uneven_row_blocks(n, k, m):
    """Shapes whose 128-row blocks would leave SMs idle without a K split: the row tiles are spread over one wave
    of blocks holding 6-8 tiles each (the box's other rows are neither decoded nor stored)."""
    import mbp
    w = weight(n, k, seed=n, escape_frac=0.01)
    p = mbp.pack_c12(w)
    x = tokens(m, k, seed=m)
    out = mbp.gemm(p, x, out_dtype=torch.float32)
    ref = torch.cat([mbp.gemv(p, x[i:i + 32].contiguous(), out_dtype=torch.float32) for i in range(0, m, 32)])
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-3)
    assert_close_bf16(mbp.gemm(p, x), ref_f32(x, w))
    assert mbp.device_status() == 0


def test_gemm_partial_rows_and_f32():
    import mbp
    w = weight(8192, 1024, seed=5, escape_frac=0.01)
    p = mbp.pack_c12(w)
    x = tokens(160, 1024, seed=6)
    out = mbp.gemm(p, x, n_out=1040)  # not a multiple of the 128-row CTA tile
    assert out.shape == (160, 1040)
    assert_close_bf16(out, ref_f32(x, w, 1040))
    o32 = mbp.gemm(p, x, out_dtype=torch.float32)
    assert torch.allclose(o32, ref_f32(x, w), rtol=1e-4, atol=1e-3)


def test_gemm_matches_gemv():
    """Both kernels compute the same FP32-accumulated products (different summation order)."""
    import mbp
    w = weight(2048, 3072, seed=8, escape_frac=0.01)
    p = mbp.pack_c12(w)
    x = tokens(32, 3072, seed=9)
    a = mbp.gemm(p, x, out_dtype=torch.float32)
    b = mbp.gemv(p, x, out_dtype=torch.float32)
    assert torch.allclose(a, b, rtol=1e-4, atol=1e-3)


def test_gemm_back_to_back_split_k_status():
    """Many back-to-back launches of a cluster split-K configuration (unpooler 1536 -> 6144, K split across CTAs)
    with no host synchronisation in between: results stay exact and no bounded wait ever gives up.  This is the
    pattern that exposed a pipeline-phase hazard when a shared-memory ring's stages alternated between the two
    decoder groups."""
    import mbp
    w = weight(6144, 1536, seed=31, escape_frac=0.01)
    p = mbp.pack_c12(w)
    copies = [p] + [mbp.PackedC12(p.units.clone(), p.bases, p.esc_off, p.esc, p.n, p.k, p.n_esc) for _ in range(3)]
    x = tokens(128, 1536, seed=32)
    ref = mbp.gemm(p, x)
    outs = [mbp.gemm(copies[i % 4], x) for i in range(64)]
    torch.cuda.synchronize()
    assert mbp.device_status() == 0
    for o in outs:
        assert torch.equal(o, ref)
    assert_close_bf16(ref, ref_f32(x, w))


@pytest.mark.parametrize("shape", [(6144, 1536), (1536, 6144), (6144, 6144)])
def test_gemm_repeated_calls_stage_reuse(shape):
    """Repeated calls at 256 tokens against the FP32 reference.  The weight producer refills a packed stage as
    soon as the decoders hand it back; a hand-back that did not wait for the decoders' shared loads to return let
    the next copy overwrite a unit under a load in flight (half a warp's rows wrong, at random, in about a third of
    the calls).  Every call must match."""
    import mbp
    n, k = shape
    w = weight(n, k, seed=41)
    p = mbp.pack_c12(w)
    x = tokens(256, k, seed=42)
    ref = ref_f32(x, w)
    outs = [mbp.gemm(p, x, out_dtype=torch.float32) for _ in range(8)]
    torch.cuda.synchronize()
    assert mbp.device_status() == 0
    for o in outs:
        assert torch.allclose(o, ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("shape,m", [((2048, 6144), 128), ((6144, 1536), 256), ((1536, 6144), 256),
                                     ((14336, 6144), 256)])
def test_gemm_deterministic(shape, m):
    """Cluster split-K partials are added in a fixed order: repeated calls give identical bits."""
    import mbp
    w = weight(*shape, seed=51, escape_frac=0.005)
    p = mbp.pack_c12(w)
    x = tokens(m, shape[1], seed=52)
    a = mbp.gemm(p, x, out_dtype=torch.float32)
    b = mbp.gemm(p, x, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert mbp.device_status() == 0
    assert torch.equal(a, b)
    assert torch.allclose(a, ref_f32(x, w), rtol=1e-3, atol=1e-2)


@pytest.mark.parametrize("layer", ["qkv_gate", "o"])
@pytest.mark.parametrize("m", [9, 16, 24, 32])
@pytest.mark.parametrize("variant", ["plain", "esc1pct"])
def test_gemm_decode_shapes(layer, m, variant):
    """The decode shapes at the token counts the tensor-core path may take."""
    import mbp
    n, k = CONFIG3[layer]
    w = weight(n, k, seed=0, escape_frac=0.01 if variant == "esc1pct" else 0.0)
    p = mbp.pack_c12(w)
    x = tokens(m, k, seed=m)
    out = mbp.gemm(p, x)
    torch.cuda.synchronize()
    assert mbp.device_status() == 0
    ref = ref_f32(x, w)
    assert_close_bf16(out, ref)
    assert_reference_norms(out, ref)


@pytest.mark.parametrize("kind", ["gather", "sum"])
@pytest.mark.parametrize("n,k,m", [(2048, 1024, 100), (1536, 6144, 256), (1024, 2048, 48)])
def test_gemm_tagged_exchange_single_rank(n, k, m, kind):
    """The GEMM's tensor-parallel epilogues (mbp_gemm_c12_multi: epoch-tagged bf16x2 words for the column gather,
    f32 words for the row-parallel sum, into the exchange buffers) read back by the receive kernel (mbp_tp_finish,
    MBP_TP_GATHER_BF16 / MBP_TP_SUM_F32) with one rank: the assembled output equals the plain GEMM bit for bit
    over three epochs (alternating buffer halves), with and without a K split."""
    import ctypes
    import mbp
    from mbp._lib import OUT_TAGGED_BF16X2, OUT_TAGGED_F32, TP_COUNTER_SLOTS, TP_GATHER_BF16, TP_SUM_F32, lib
    from mbp.ops import _stream
    w = weight(n, k, seed=3, escape_frac=0.01)
    p = mbp.pack_c12(w)
    gather = kind == "gather"
    ldo = n // 2 if gather else n
    par = -(-(m * ldo * 8) // 256) * 256
    buf = torch.zeros(2 * par, dtype=torch.uint8, device="cuda")
    counter = torch.zeros(TP_COUNTER_SLOTS + 1, dtype=torch.int32, device="cuda")
    outs = (ctypes.c_void_p * 1)(buf.data_ptr())
    for i in range(3):
        x = tokens(m, k, seed=10 + i)
        out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        rc = lib().mbp_gemm_c12_multi(ctypes.byref(p.desc), x.data_ptr(), m, n, outs, 1, ldo,
                                      OUT_TAGGED_BF16X2 if gather else OUT_TAGGED_F32, counter.data_ptr(), par,
                                      _stream())
        assert rc == 0, rc
        rc = lib().mbp_tp_finish(None, 0, 1, counter.data_ptr(), buf.data_ptr(), par,
                                 TP_GATHER_BF16 if gather else TP_SUM_F32, m, n, out.data_ptr(), _stream())
        assert rc == 0, rc
        assert torch.equal(out, mbp.gemm(p, x)), i
    assert int(counter[0]) == 3
    assert mbp.device_status() == 0
