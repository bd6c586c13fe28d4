"""Pins the CPU oracle against golden vectors produced by the reference's own functions.

Fixtures: ``tests/golden/*.npz`` and ``golden_summary.json``, written by ``tests/golden/make_golden.py`` which
imports the reference's ``sm_units`` / ``sm_c12_bytes`` / ``sm_c12_unpack`` / ``sm_table`` / ``sm_bf16_bytes`` /
``sm_pack_format`` (submission.py:82-176).
"""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import c12

CASES = ["c12_n64_k256", "c12_n32_k512_esc", "c12_n48_k192_wide"]


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def ref_esc(g):
    return {"r": g["esc_r"], "c": g["esc_c"], "lane": g["esc_lane"], "v": g["esc_v"], "xor7": g["esc_xor7"]}


@pytest.mark.parametrize("name", CASES)
def test_units_match_reference(name):
    g = load(name)
    u = c12.units(g["w"])
    assert np.array_equal(u, g["units"].astype(np.int64) & 0xFFFF)
    assert np.array_equal(c12.from_units(u), g["w"])


@pytest.mark.parametrize("name", CASES)
def test_pack_matches_reference_bytes(name):
    g = load(name)
    data, bases, esc = c12.c12_pack(c12.units(g["w"]), "matrix")
    assert int(bases[0]) == int(g["base"]) and np.all(bases == bases[0])
    assert np.array_equal(data, g["data"])
    for key, gk in (("r", "esc_r"), ("c", "esc_c"), ("lane", "esc_lane"), ("v", "esc_v"), ("xor7", "esc_xor7")):
        assert np.array_equal(esc[key], g[gk]), key


@pytest.mark.parametrize("name", CASES)
def test_unpack_inverts_reference_pack(name):
    g = load(name)
    bases = np.full(g["data"].shape[0], int(g["base"]), dtype=np.uint8)
    u = c12.c12_unpack(g["data"], bases, ref_esc(g))
    assert np.array_equal(u, g["units"].astype(np.int64) & 0xFFFF)


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("mode", ["matrix", "tile"])
def test_csr_round_trip(name, mode):
    g = load(name)
    p = c12.pack_matrix(g["w"], mode)
    assert np.array_equal(c12.unpack_matrix(p), g["w"])
    if mode == "tile":
        # per-tile bases never need more escapes than the single matrix base
        assert p["esc"].size <= g["esc_r"].size


@pytest.mark.parametrize("name", CASES)
def test_table_matches_reference(name):
    g = load(name)
    t0, t1 = c12.decode_table(int(g["base"]))
    v = t0 | t1 << 32
    assert (v - 2**64 if v >= 2**63 else v) == int(g["table"])


@pytest.mark.parametrize("name", CASES)
def test_raw_units_match_reference(name):
    g = load(name)
    assert np.array_equal(c12.raw_units(g["w"]), g["bf16_bytes"])


@pytest.mark.parametrize("name", CASES)
def test_register_decode_model(name):
    """The prmt-level decode model (what the CUDA kernel does) reproduces the units exactly."""
    g = load(name)
    p = c12.pack_matrix(g["w"], "tile")
    u = c12.units(g["w"])
    r, c = u.shape[:2]
    for ri in range(r):
        for ci in range(c):
            ui = ri * c + ci
            ents = p["esc"][p["esc_off"][ui]:p["esc_off"][ui + 1]]
            regs = c12.decode_unit(p["units"][ri, ci], int(p["bases"][ri]), [int(e) for e in ents])
            vals = np.stack([regs & 0xFFFF, regs >> 16], axis=-1).reshape(32, 32)
            assert np.array_equal(vals.astype(np.int64), u[ri, ci]), (ri, ci)


def test_verify_vectors_linear():
    """FP64 reference outputs of the reference's random + spike recipe (S:297-317), rounded to BF16."""
    g = load("c12_n64_k256")
    for i in range(3):
        out = c12.linear(g[f"x{i}"], g["w"], acc="f64")
        assert np.array_equal(c12.f32_to_bf16_bits(out), g[f"ref{i}"])


def test_router_hilo_matches_reference():
    g = load("router_n32_k128")
    hi, lo = c12.router_hilo(g["w"])
    assert np.array_equal(hi, g["hi"]) and np.array_equal(lo, g["lo"])
    exact = c12.bf16_bits_to_f32(hi) + c12.bf16_bits_to_f32(lo)
    assert np.array_equal(exact, g["exact"])
    assert np.array_equal(np.concatenate([c12.raw_units(hi), c12.raw_units(lo)], axis=-1), g["data"])
    for i in range(2):
        got = c12.linear(g[f"x{i}"], hi, "f64").astype(np.float64) + c12.linear(g[f"x{i}"], lo, "f64")
        ref = g[f"ref{i}"].astype(np.float64)
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5


def test_bf16_rounding():
    vals = np.array([1.0, 1.00390625, 1.0078125, -2.5, 3.1415926, 1e-40, np.inf, -np.inf], dtype=np.float32)
    import torch
    want = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(c12.f32_to_bf16_bits(vals), want)


@pytest.mark.slow
def test_config1_known_answer():
    """The reference's CPU-runnable case (4096 x 4096, N(0, 0.02), torch seed 0): its base, escape count and packed
    bytes (sha256) are reproduced by the oracle."""
    import torch
    s = json.load(open(os.path.join(GOLDEN, "golden_summary.json")))["config1_4096x4096"]
    torch.manual_seed(0)
    w = (torch.randn(4096, 4096) * 0.02).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert hashlib.sha256(w.tobytes()).hexdigest() == s["w_sha256"]
    data, bases, esc = c12.c12_pack(c12.units(w), "matrix")
    assert int(bases[0]) == s["base"] and esc["r"].size == s["n_esc"]
    assert hashlib.sha256(data.tobytes()).hexdigest() == s["data_sha256"]
    e = np.stack([esc[k] for k in ("r", "c", "lane", "v", "xor7")]).astype(np.int64)
    assert hashlib.sha256(e.tobytes()).hexdigest() == s["esc_sha256"]
