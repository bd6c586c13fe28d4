"""Packed on-disk format (mbp.store) on the host: byte-exact round trips of c12 and hi/lo layers (packed by the
oracle), fingerprints, and rejection of files that are not, or no longer, what the caller's weights describe."""
import numpy as np
import pytest
import torch

from mbp import store
from mbp.ops import PackedC12, PackedHiLo
from oracle import oracle


def _c12_state(seed=0, n=64, k=256):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.02)
    w.view(-1)[torch.randperm(n * k, generator=g)[: n * k // 50]] *= 256  # escapes
    w = w.to(torch.bfloat16)
    p = oracle.pack(w.view(torch.int16).numpy().view(np.uint16), tile_base=True)
    pc = PackedC12(torch.from_numpy(p["units"]), torch.from_numpy(p["bases"]), torch.from_numpy(p["esc_off"]),
                   torch.from_numpy(p["esc"].view(np.int32)), n, k, int(p["esc"].size))
    units = torch.randint(0, 256, (1, 4, 2, 2048), dtype=torch.uint8, generator=g)
    ph = PackedHiLo(units, 16, 256)
    return w, p, {"layers": {"o": pc}, "hilo": {"router": ph}, "k": {"o": k, "router": 256}}


def test_round_trip_is_byte_exact(tmp_path):
    w, p, st = _c12_state()
    assert st["layers"]["o"].n_esc > 0
    path = str(tmp_path / "w.mbp")
    fps = {"o": store.fingerprint(w), "router": "r"}
    store.save_packed(st, path, fps, base_mode=1)
    back = store.load_packed(path, device="cpu")
    a, b = st["layers"]["o"], back["layers"]["o"]
    assert (a.n, a.k, a.n_esc) == (b.n, b.k, b.n_esc)
    for name in ("units", "bases", "esc_off", "esc"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    assert torch.equal(st["hilo"]["router"].units, back["hilo"]["router"].units)
    assert back["k"] == {"o": 256, "router": 256}
    # the reloaded layer still unpacks to the original weights (oracle restatement of the format)
    q = {"n": b.n, "k": b.k, "units": b.units.numpy(), "bases": b.bases.numpy(), "esc_off": b.esc_off.numpy(),
         "esc": b.esc.numpy().view(np.uint32)}
    assert np.array_equal(oracle.unpack(q), w.view(torch.int16).numpy().view(np.uint16))
    assert store.matches(path, fps, 1)
    assert not store.matches(path, fps, 0)                      # other base mode
    assert not store.matches(path, {"o": fps["o"]}, 1)          # other layer set
    assert not store.matches(path, {"o": "x", "router": "r"}, 1)  # other weights


def test_layer_without_escapes(tmp_path):
    n, k = 32, 128
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(3)) * 0.02).to(torch.bfloat16)
    p = oracle.pack(w.view(torch.int16).numpy().view(np.uint16), tile_base=False)
    esc = torch.from_numpy(p["esc"].view(np.int32))
    pc = PackedC12(torch.from_numpy(p["units"]), torch.from_numpy(p["bases"]), torch.from_numpy(p["esc_off"]), esc,
                   n, k, int(esc.numel()))
    path = str(tmp_path / "w.mbp")
    store.save_packed({"layers": {"q": pc}, "hilo": {}, "k": {"q": k}}, path, {"q": "f"}, base_mode=0)
    back = store.load_packed(path, device="cpu")["layers"]["q"]
    assert back.n_esc == pc.n_esc and torch.equal(back.esc, pc.esc) and torch.equal(back.units, pc.units)


def test_fingerprint_sees_any_element():
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(256, 512, generator=g) * 0.02).to(torch.bfloat16)
    f0 = store.fingerprint(w)
    assert store.fingerprint(w.clone()) == f0
    for i in (0, 1, 7, 12345, w.numel() - 1):  # sampled and unsampled positions
        v = w.clone()
        v.view(-1)[i] = -v.view(-1)[i] if float(v.view(-1)[i]) != 0 else 1.0
        assert store.fingerprint(v) != f0, i
    assert store.fingerprint(w.reshape(512, 256)) != f0
    assert store.fingerprint(w.float()) != f0


def test_rejects_foreign_and_truncated_files(tmp_path):
    bad = tmp_path / "bad.mbp"
    bad.write_bytes(b"NOTAPACK" + b"\0" * 64)
    with pytest.raises(ValueError):
        store.read_header(str(bad))
    assert not store.matches(str(bad), {}, 1)
    assert not store.matches(str(tmp_path / "missing.mbp"), {}, 1)
    _, _, st = _c12_state(seed=1)
    path = tmp_path / "w.mbp"
    store.save_packed(st, str(path), {"o": "a", "router": "b"}, base_mode=1)
    data = path.read_bytes()
    path.write_bytes(data[: len(data) - 5000])
    with pytest.raises(ValueError):
        store.load_packed(str(path), device="cpu")
