"""The C port of the oracle agrees bit for bit with the numpy restatement (itself pinned by test_oracle.py)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import c12, oracle

CASES = ["c12_n64_k256", "c12_n32_k512_esc", "c12_n48_k192_wide"]


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("tile", [False, True])
def test_c_pack_equals_numpy(name, tile):
    g = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    a = oracle.pack(g["w"], tile_base=tile)
    b = c12.pack_matrix(g["w"], "tile" if tile else "matrix")
    for key in ("units", "bases", "esc_off", "esc"):
        assert np.array_equal(a[key], b[key]), key
    assert np.array_equal(oracle.unpack(a), g["w"])
    if not tile:
        assert np.array_equal(a["units"], g["data"])


@pytest.mark.parametrize("name", ["c12_n64_k256", "c12_n32_k512_esc"])
def test_c_gemv_matches_f64(name):
    g = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    p = oracle.pack(g["w"], True)
    rng = np.random.default_rng(0)
    x = c12.f32_to_bf16_bits(rng.standard_normal((5, g["w"].shape[1])).astype(np.float32))
    of, ob = oracle.gemv_packed(x, p)
    ref = oracle.linear_f64(x, g["w"])
    assert np.allclose(of, ref, rtol=1e-5, atol=1e-5)
    assert np.array_equal(ob, c12.f32_to_bf16_bits(of))


def test_c_gemv_row_sample():
    g = dict(np.load(os.path.join(GOLDEN, "c12_n64_k256.npz")))
    p = oracle.pack(g["w"], True)
    x = g["x1"]
    full, _ = oracle.gemv_packed(x, p)
    part, _ = oracle.gemv_packed(x, p, row0=16, nrows=32)
    assert np.array_equal(part[:, 16:48], full[:, 16:48])
    assert not part[:, :16].any() and not part[:, 48:].any()
