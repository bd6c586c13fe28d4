"""CPU oracle (numpy) for the 12-bit lossless BF16 weight format and the small-M projection.

TEST INFRASTRUCTURE ONLY.  Nothing on the product path imports this module: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may use
it, and only as the checker.  The product path (``mbp``) runs hand-written CUDA and fails loudly when the
CUDA library is missing.

It restates, in plain numpy, the algorithm of the reference submission (NathenFernandes/muse-bf16-proj,
``submission.py``; cited as ``S:<line>``; ``S:46<a-b>`` means lines a-b of the CUDA text stored compressed on
line 46):

* ``units``          -- BF16 [N, K] -> 16x64 units in mma.sync A-fragment order          (S:82-87)
* ``c12_pack``       -- units -> 1536-byte 12-bit units, exponent base, escape list        (S:104-125)
* ``c12_unpack``     -- exact inverse                                                      (S:128-142)
* ``decode_table``   -- the prmt byte table ``base .. base+7``                             (S:145-149)
* ``decode_unit``    -- bit-level model of the in-register decode + escape patch
                        (S:46<43-51> sm_dec, S:46<155-162> sm_patch)
* ``linear``         -- ``x @ W.T`` with FP32 (or FP64) accumulation, BF16 round-to-nearest-even output
                        (the semantics of S:2610-2617 and the FP64 check of S:297-317)
* ``router_hilo``    -- FP32 weight -> (hi, lo) BF16 pair, hi = bf16(w), lo = bf16(w - hi)   (S:876-879)

Parity is pinned: ``tests/golden/`` holds vectors produced by importing the reference's own functions
(``tests/golden/make_golden.py``), and ``tests/test_oracle.py`` checks this module against them bit for bit.

Two generalisations beyond the reference, both reducing to it exactly:

* ``base_mode="matrix"`` reproduces the reference's single per-matrix exponent base, byte for byte.
  ``base_mode="tile"`` picks one base per 16-row tile with the same window rule.
* Escapes are returned both in the reference's ``(r, c, lane, value, xor7)`` form and in this build's
  compressed-sparse form: ``esc_off[r*C + c]`` offsets and 32-bit entries
  ``c << 17 | lane << 12 | value << 7 | xor7`` sorted by (r, c, lane, value) -- no per-warp cap.
"""
from __future__ import annotations

import numpy as np

UNIT_ROWS = 16
UNIT_COLS = 64
UNIT_BYTES = 1536          # 1024 weights x 12 bits
RAW_UNIT_BYTES = 2048      # 1024 weights x 16 bits (hi/lo router planes)
SIGN_POS = (3, 19, 7, 23, 11, 27, 15, 31)   # S:58: sign bit of value i inside a code word
MAX_CHUNKS = 1 << 15       # escape entry keeps 15 bits of chunk index


# ----------------------------------------------------------------------------------------------------------
# bf16 helpers
# ----------------------------------------------------------------------------------------------------------
def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even FP32 -> BF16 bit patterns (uint16); NaN kept quiet."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(a)
    out = rounded.astype(np.uint16)
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------------------------------------
# layout: S:82-87
# ----------------------------------------------------------------------------------------------------------
def units(w_bits: np.ndarray) -> np.ndarray:
    """BF16 bits [N, K] -> int64 [N/16, K/64, 32 lanes, 32 values] in mma.sync A-fragment order.

    Lane l = 4*g + t and value v = 8*q + 4*hf + 2*rh + d hold the weight at
    row 8*rh + g, column 16*t + 4*q + 2*hf + d of the 16x64 unit (S:84-86)."""
    n, k = w_bits.shape
    assert n % UNIT_ROWS == 0 and k % UNIT_COLS == 0, (n, k)
    v = w_bits.astype(np.int64).reshape(n // 16, 2, 8, k // 64, 4, 4, 2, 2).transpose(0, 3, 2, 4, 5, 6, 1, 7)
    return np.ascontiguousarray(v.reshape(n // 16, k // 64, 32, 32))


def from_units(u: np.ndarray) -> np.ndarray:
    """Inverse of ``units``."""
    r, c = u.shape[:2]
    v = u.reshape(r, c, 8, 4, 4, 2, 2, 2).transpose(0, 6, 2, 1, 3, 4, 5, 7)
    return np.ascontiguousarray(v.reshape(r * 16, c * 64)).astype(np.uint16)


# ----------------------------------------------------------------------------------------------------------
# 12-bit packing: S:104-125 (pack), S:128-142 (unpack)
# ----------------------------------------------------------------------------------------------------------
def window_base(hist: np.ndarray) -> int:
    """argmax over b in [0, 121) of sum(hist[b:b+8]), first maximum wins (S:111-113)."""
    csum = np.concatenate([[0], np.cumsum(hist.astype(np.int64))])
    window = csum[8:129] - csum[0:121]
    return int(np.argmax(window))


def c12_pack(u: np.ndarray, base_mode: str = "matrix"):
    """Units -> (data uint8 [R, C, 1536], bases uint8 [R], escapes dict).

    data plane 0 = lane-major low bytes of values 0-15, plane 1 = values 16-31, plane 2 = four little-endian
    code words per lane, word w holding values 8w..8w+7 as 3-bit exponent offsets at nibble i and the sign at
    bit SIGN_POS[i] (S:114-121)."""
    r, c = u.shape[:2]
    lo = (u & 0xFF).astype(np.uint8)
    sign = (u >> 15) & 1
    eh = (u >> 8) & 0x7F
    if base_mode == "matrix":
        b = window_base(np.bincount(eh.reshape(-1), minlength=128))
        bases = np.full(r, b, dtype=np.int64)
    elif base_mode == "tile":
        bases = np.array([window_base(np.bincount(eh[i].reshape(-1), minlength=128)) for i in range(r)],
                         dtype=np.int64)
    else:
        raise ValueError(base_mode)
    bb = bases[:, None, None, None]
    d = eh - bb
    inwin = (d >= 0) & (d < 8)
    d = np.where(inwin, d, 0)
    nib = np.arange(8, dtype=np.int64) * 4
    pos = np.array(SIGN_POS, dtype=np.int64)
    code = ((d.reshape(r, c, 32, 4, 8) << nib) + (sign.reshape(r, c, 32, 4, 8) << pos)).sum(-1)
    code_bytes = code.astype(np.uint32).view(np.uint8).reshape(r, c, 32, 16)
    data = np.stack([lo[..., :16], lo[..., 16:], code_bytes], axis=2).reshape(r, c, UNIT_BYTES)
    er, ec, el, ev = np.nonzero(~inwin)
    xor7 = eh[er, ec, el, ev] ^ bases[er]
    esc = {"r": er.astype(np.int64), "c": ec.astype(np.int64), "lane": el.astype(np.int64),
           "v": ev.astype(np.int64), "xor7": xor7.astype(np.int64)}
    return np.ascontiguousarray(data), bases.astype(np.uint8), esc


def c12_unpack(data: np.ndarray, bases: np.ndarray, esc: dict) -> np.ndarray:
    """Exact inverse of ``c12_pack`` (S:128-142)."""
    r, c = data.shape[:2]
    p = data.reshape(r, c, 3, 32, 16)
    lo = np.concatenate([p[:, :, 0], p[:, :, 1]], axis=-1).astype(np.int64)
    code = np.ascontiguousarray(p[:, :, 2]).view(np.uint32).reshape(r, c, 32, 4).astype(np.int64)
    nib = np.arange(8, dtype=np.int64) * 4
    pos = np.array(SIGN_POS, dtype=np.int64)
    d = ((code[..., None] >> nib) & 7).reshape(r, c, 32, 32)
    sg = ((code[..., None] >> pos) & 1).reshape(r, c, 32, 32)
    base = bases.astype(np.int64)[:, None, None, None]
    val = (sg << 15) | ((base + d) << 8) | lo
    val[esc["r"], esc["c"], esc["lane"], esc["v"]] ^= esc["xor7"] << 8
    return val


def escapes_csr(esc: dict, r: int, c: int):
    """Reference-form escape list -> (esc_off int32 [R*C+1], entries uint32 [E]) sorted by (r, c, lane, v)."""
    assert c < MAX_CHUNKS
    key = ((esc["r"] * c + esc["c"]) * 32 + esc["lane"]) * 32 + esc["v"]
    order = np.argsort(key, kind="stable")
    ur = esc["r"][order] * c + esc["c"][order]
    entries = ((esc["c"][order] << 17) | (esc["lane"][order] << 12) | (esc["v"][order] << 7)
               | esc["xor7"][order]).astype(np.uint32)
    counts = np.bincount(ur, minlength=r * c)
    off = np.zeros(r * c + 1, dtype=np.int64)
    np.cumsum(counts, out=off[1:])
    return off.astype(np.int32), entries


def escapes_from_csr(off: np.ndarray, entries: np.ndarray, r: int, c: int) -> dict:
    """CSR escape list -> reference form."""
    e = entries.astype(np.int64)
    unit = np.repeat(np.arange(r * c, dtype=np.int64), np.diff(off.astype(np.int64)))
    return {"r": unit // c, "c": (e >> 17) & 0x7FFF, "lane": (e >> 12) & 31, "v": (e >> 7) & 31, "xor7": e & 0x7F}


def pack_matrix(w_bits: np.ndarray, base_mode: str = "matrix") -> dict:
    """BF16 bits [N, K] -> the full packed description used by this build."""
    n, k = w_bits.shape
    u = units(w_bits)
    data, bases, esc = c12_pack(u, base_mode)
    off, entries = escapes_csr(esc, n // 16, k // 64)
    return {"n": n, "k": k, "units": data, "bases": bases, "esc_off": off, "esc": entries}


def unpack_matrix(p: dict) -> np.ndarray:
    r, c = p["n"] // 16, p["k"] // 64
    esc = escapes_from_csr(p["esc_off"], p["esc"], r, c)
    return from_units(c12_unpack(p["units"], p["bases"], esc))


# ----------------------------------------------------------------------------------------------------------
# bit-level model of the in-register decode: S:145-149 (table), S:46<43-51> (sm_dec), S:46<155-162> (patch)
# ----------------------------------------------------------------------------------------------------------
def decode_table(base: int) -> tuple[int, int]:
    t0 = base | (base + 1) << 8 | (base + 2) << 16 | (base + 3) << 24
    t1 = (base + 4) | (base + 5) << 8 | (base + 6) << 16 | (base + 7) << 24
    return t0, t1


def prmt(a: int, b: int, sel: int) -> int:
    """PTX prmt.b32 default mode: byte i of the result is byte (sel nibble i & 7) of {b, a}, sign-replicated
    when bit 3 of the nibble is set."""
    src = (a & 0xFFFFFFFF) | (b & 0xFFFFFFFF) << 32
    out = 0
    for i in range(4):
        s = (sel >> (4 * i)) & 0xF
        byte = (src >> (8 * (s & 7))) & 0xFF
        if s & 8:
            byte = 0xFF if byte & 0x80 else 0
        out |= byte << (8 * i)
    return out


def decode_group(l0: int, l1: int, code: int, t0: int, t1: int) -> list[int]:
    """8 weights of one k16 step -> 4 packed bf16x2 A registers."""
    cm = code & 0x77777777
    hlo = prmt(t0, t1, cm & 0xFFFF)
    hhi = prmt(t0, t1, (cm >> 16) & 0xFFFF)
    return [prmt(l0, hlo, 0x5140) | ((code << 12) & 0x80008000),
            prmt(l0, hlo, 0x7362) | ((code << 8) & 0x80008000),
            prmt(l1, hhi, 0x5140) | ((code << 4) & 0x80008000),
            prmt(l1, hhi, 0x7362) | (code & 0x80008000)]


def decode_unit(unit_bytes: np.ndarray, base: int, entries=()) -> np.ndarray:
    """One 1536-byte unit -> uint32 [32 lanes, 16 registers] exactly as the GEMV holds them in registers."""
    t0, t1 = decode_table(base)
    p = unit_bytes.reshape(3, 32, 16)
    regs = np.zeros((32, 16), dtype=np.uint64)
    for lane in range(32):
        lo = np.concatenate([p[0, lane], p[1, lane]]).view(np.uint32)   # 8 words: 4 values each
        code = p[2, lane].view(np.uint32)
        for q in range(4):
            a = decode_group(int(lo[2 * q]), int(lo[2 * q + 1]), int(code[q]), t0, t1)
            regs[lane, 4 * q:4 * q + 4] = a
    for e in entries:
        lane, v, x7 = (e >> 12) & 31, (e >> 7) & 31, e & 0x7F
        regs[lane, v >> 1] ^= x7 << (8 + 16 * (v & 1))
    return regs.astype(np.uint32)


# ----------------------------------------------------------------------------------------------------------
# arithmetic: the projection and the router split
# ----------------------------------------------------------------------------------------------------------
def linear(x_bits: np.ndarray, w_bits: np.ndarray, acc: str = "f32") -> np.ndarray:
    """out[M, N] = x[M, K] . W[N, K]^T from BF16 bit patterns, FP32 (or FP64) accumulation, FP32 result."""
    x = bf16_bits_to_f32(x_bits)
    w = bf16_bits_to_f32(w_bits)
    if acc == "f64":
        return (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)
    return (x @ w.T).astype(np.float32)


def router_hilo(w_f32: np.ndarray):
    """FP32 weight -> (hi, lo) BF16 bit patterns with hi + lo ~= w to 16 significant bits (S:876-879)."""
    w = np.ascontiguousarray(w_f32, dtype=np.float32)
    hi = f32_to_bf16_bits(w)
    lo = f32_to_bf16_bits(w - bf16_bits_to_f32(hi))
    return hi, lo


def raw_units(w_bits: np.ndarray) -> np.ndarray:
    """BF16 bits [N, K] -> uint8 [N/16, K/64, 2048]: the unit values stored uncompressed, laid out as four
    512-byte lane-major planes of 8 values each (S:98-101 ``sm_bf16_bytes``)."""
    u = units(w_bits)
    r, c = u.shape[:2]
    words = u.reshape(r, c, 32, 4, 8).transpose(0, 1, 3, 2, 4).astype(np.uint16)
    return np.ascontiguousarray(words).view(np.uint8).reshape(r, c, RAW_UNIT_BYTES)
