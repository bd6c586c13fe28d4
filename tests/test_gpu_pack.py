"""GPU packer parity: bytes, bases and escape lists identical to the oracle (and, in matrix-base mode, to the
reference's own packer output stored in tests/golden); device unpack is the exact inverse."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import bits_np, weight
from oracle import c12, oracle

pytestmark = pytest.mark.gpu

CASES = ["c12_n64_k256", "c12_n32_k512_esc", "c12_n48_k192_wide"]


def to_dev_bf16(wbits):
    return torch.from_numpy(wbits.astype(np.int16)).view(torch.bfloat16).cuda()


def packed_np(p):
    return {"units": p.units.cpu().numpy(), "bases": p.bases.cpu().numpy(), "esc_off": p.esc_off.cpu().numpy(),
            "esc": p.esc.cpu().numpy().view(np.uint32)}


@pytest.mark.parametrize("name", CASES)
def test_matrix_mode_equals_reference_bytes(name):
    import mbp
    g = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    p = mbp.pack_c12(to_dev_bf16(g["w"]), mbp.BASE_MATRIX)
    got = packed_np(p)
    assert np.array_equal(got["units"], g["data"])
    assert np.all(got["bases"] == int(g["base"]))
    esc = c12.escapes_from_csr(got["esc_off"], got["esc"], got["units"].shape[0], got["units"].shape[1])
    for key, gk in (("r", "esc_r"), ("c", "esc_c"), ("lane", "esc_lane"), ("v", "esc_v"), ("xor7", "esc_xor7")):
        assert np.array_equal(esc[key], g[gk]), key
    assert mbp.device_status() == 0


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("mode", [0, 1])
def test_pack_equals_oracle_and_round_trips(name, mode):
    import mbp
    g = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    w = to_dev_bf16(g["w"])
    p = mbp.pack_c12(w, mode)
    ref = oracle.pack(g["w"], tile_base=bool(mode))
    got = packed_np(p)
    for key in ("units", "bases", "esc_off", "esc"):
        assert np.array_equal(got[key], ref[key]), key
    back = mbp.unpack_c12(p)
    assert torch.equal(back.view(torch.int16), w.view(torch.int16))


@pytest.mark.parametrize("shape,frac", [((1536, 6144), 0.0), ((6144, 1536), 0.01), ((4096, 4096), 0.0),
                                        ((256, 6144), 0.01)])
def test_pack_large_against_c_oracle(shape, frac):
    import mbp
    w = weight(*shape, seed=0, escape_frac=frac)
    p = mbp.pack_c12(w, mbp.BASE_TILE)
    ref = oracle.pack(bits_np(w), tile_base=True)
    got = packed_np(p)
    for key in ("units", "bases", "esc_off", "esc"):
        assert np.array_equal(got[key], ref[key]), key
    assert torch.equal(mbp.unpack_c12(p).view(torch.int16), w.view(torch.int16))


@pytest.mark.parametrize("shape", [(14336, 6144), (6144, 6144)])
@pytest.mark.parametrize("frac", [0.0, 0.01])
def test_round_trip_baseline_shapes(shape, frac):
    """Full benchmark shapes: device round trip bit-exact; escape count equals the oracle's count."""
    import mbp
    w = weight(*shape, seed=0, escape_frac=frac)
    p = mbp.pack_c12(w, mbp.BASE_TILE)
    assert torch.equal(mbp.unpack_c12(p).view(torch.int16), w.view(torch.int16))
    ref = oracle.pack(bits_np(w), tile_base=True)
    assert p.n_esc == ref["esc"].size
    assert np.array_equal(p.bases.cpu().numpy(), ref["bases"])


def test_special_values_round_trip():
    """Zeros, signed zeros, subnormals, infinities, NaNs and every exponent survive the round trip."""
    import mbp
    vals = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    w = torch.from_numpy(vals.astype(np.int16)).view(torch.bfloat16).reshape(64, 1024).cuda()
    for mode in (0, 1):
        p = mbp.pack_c12(w, mode)
        assert torch.equal(mbp.unpack_c12(p).view(torch.int16), w.view(torch.int16))


def test_hilo_pack_matches_reference():
    import mbp
    g = dict(np.load(os.path.join(GOLDEN, "router_n32_k128.npz")))
    p = mbp.pack_hilo(torch.from_numpy(g["w"]).cuda())
    got = p.units.cpu().numpy().reshape(2, 2, 2, 2048)  # [r, c, half, bytes]
    ref = g["data"].reshape(2, 2, 2, 2048)  # reference fmt 2: hi unit bytes then lo unit bytes
    assert np.array_equal(got, ref)
