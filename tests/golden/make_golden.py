"""Generates the golden fixtures in this directory from the reference's OWN functions.

Run once, in a container that has the reference checkout (path given by ``--reference``):

    python tests/golden/make_golden.py --reference <path to muse-bf16-proj checkout>

It imports the reference's ``submission.py`` with a stub for the ``sglang`` module (only its GPU fallback uses
it, S:18 / S:2610-2617), then calls the reference's packing functions on CPU tensors:

* ``sm_units`` (S:82-87), ``sm_c12_bytes`` (S:104-125), ``sm_c12_unpack`` (S:128-142), ``sm_table``
  (S:145-149), ``sm_bf16_bytes`` (S:98-101), ``sm_pack_format`` (S:152-176, router hi/lo fmt 2).
* The random-plus-spike input recipe of ``sm_verify_random`` (S:297-317) and its FP64 reference output.

Nothing under ``tests/`` reads the reference at run time; the tests only read the ``.npz`` / ``.json`` files
written here.  Inputs are seeded synthetic tensors (the reference ships no stored vectors).
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(path: str):
    # The reference imports sglang at module top for its GPU fallback; a stub is enough for the packers.
    for name in ("sglang", "sglang.srt", "sglang.srt.layers", "sglang.srt.layers.quantization",
                 "sglang.srt.layers.quantization.unquant"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["sglang.srt.layers.quantization.unquant"]._bf16_gemm_dispatch_impl = None
    spec = importlib.util.spec_from_file_location("ref_submission", os.path.join(path, "submission.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def packed_case(ref, w: torch.Tensor):
    u = ref.sm_units(w)
    data, base, esc = ref.sm_c12_bytes(u)
    back = ref.sm_c12_unpack(data, base, esc)
    assert torch.equal(back, u), "reference round trip failed"
    er, ec, el, ev, x7 = esc
    return {
        "w": bits(w),
        "units": u.numpy().astype(np.int32),
        "data": data.numpy().astype(np.uint8),
        "base": np.array(base, dtype=np.int64),
        "esc_r": er.numpy().astype(np.int64), "esc_c": ec.numpy().astype(np.int64),
        "esc_lane": el.numpy().astype(np.int64), "esc_v": ev.numpy().astype(np.int64),
        "esc_xor7": x7.numpy().astype(np.int64),
        "table": np.array(ref.sm_table(base), dtype=np.int64),
        "bf16_bytes": ref.sm_bf16_bytes(u).numpy().astype(np.uint8),
    }


def verify_inputs(w: torch.Tensor, ms, seed=11):
    """The reference's random + spike recipe (S:305-310) and FP64 reference rounded to BF16 (S:310)."""
    n, k = w.shape
    gen = torch.Generator().manual_seed(seed)
    xs, refs = [], []
    for m in ms:
        x = torch.randn((m, k), generator=gen)
        x[m - 1].zero_()
        x[m - 1, (seed * 131 + m) % k] = 16.0
        x = x.to(torch.bfloat16)
        ref = (x.double() @ w.double().T).to(torch.bfloat16)
        xs.append(bits(x))
        refs.append(bits(ref))
    return xs, refs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    ref = load_reference(args.reference)
    assert ref.SM_SIGN_POS == (3, 19, 7, 23, 11, 27, 15, 31)
    summary = {"generator": "tests/golden/make_golden.py", "cases": {}}

    # 1. small N(0, 0.02) matrix, the benchmark's weight distribution
    torch.manual_seed(0)
    w = (torch.randn(64, 256) * 0.02).to(torch.bfloat16)
    case = packed_case(ref, w)
    xs, refs = verify_inputs(w, (1, 5, 8))
    for i, (x, r) in enumerate(zip(xs, refs)):
        case[f"x{i}"], case[f"ref{i}"] = x, r
    np.savez_compressed(os.path.join(HERE, "c12_n64_k256.npz"), **case)
    summary["cases"]["c12_n64_k256"] = {"base": int(case["base"]), "n_esc": int(case["esc_r"].size)}

    # 2. escape stress: 1% of weights scaled x256 (the benchmark's escape variant, small)
    torch.manual_seed(0)
    w = (torch.randn(32, 512) * 0.02)
    idx = torch.randperm(w.numel(), generator=torch.Generator().manual_seed(2))[: w.numel() // 100]
    w.view(-1)[idx] *= 256
    w = w.to(torch.bfloat16)
    case = packed_case(ref, w)
    np.savez_compressed(os.path.join(HERE, "c12_n32_k512_esc.npz"), **case)
    summary["cases"]["c12_n32_k512_esc"] = {"base": int(case["base"]), "n_esc": int(case["esc_r"].size)}

    # 3. wide dynamic range (many escapes, zeros, subnormals, infinities and a NaN)
    g = torch.Generator().manual_seed(3)
    w = torch.randn(48, 192, generator=g) * torch.exp2(torch.randint(-30, 30, (48, 192), generator=g).float())
    w[0, :8] = 0.0
    w[1, :4] = torch.tensor([1e-40, -1e-41, float("inf"), float("-inf")])
    w[2, 0] = float("nan")
    w = w.to(torch.bfloat16)
    case = packed_case(ref, w)
    np.savez_compressed(os.path.join(HERE, "c12_n48_k192_wide.npz"), **case)
    summary["cases"]["c12_n48_k192_wide"] = {"base": int(case["base"]), "n_esc": int(case["esc_r"].size)}

    # 4. router: FP32 weights split into hi/lo BF16 planes (fmt 2, S:152-160)
    torch.manual_seed(4)
    wr = torch.randn(32, 128) * 0.01
    pk = ref.sm_pack_format(wr, 2)
    hi = wr.to(torch.bfloat16)
    lo = (wr - hi.float()).to(torch.bfloat16)
    xs, refs = [], []
    gen = torch.Generator().manual_seed(11)
    for m in (1, 4):
        x = torch.randn((m, 128), generator=gen).to(torch.bfloat16)
        xs.append(bits(x))
        refs.append((x.double() @ wr.double().T).to(torch.float32).numpy())
    np.savez_compressed(os.path.join(HERE, "router_n32_k128.npz"), w=wr.numpy(), hi=bits(hi), lo=bits(lo),
                        data=pk["data"].numpy().astype(np.uint8),
                        exact=ref.sm_exact(wr, 2).numpy(), x0=xs[0], x1=xs[1], ref0=refs[0], ref1=refs[1])

    # 5. known answers on the reference's CPU-runnable matrix (4096 x 4096, N(0, 0.02), torch seed 0): too large to
    #    store, so the fixture keeps the reference's base, escape count and sha256 of its packed bytes.
    torch.manual_seed(0)
    w = (torch.randn(4096, 4096) * 0.02).to(torch.bfloat16)
    u = ref.sm_units(w)
    data, base, esc = ref.sm_c12_bytes(u)
    assert torch.equal(ref.sm_c12_unpack(data, base, esc), u)
    summary["config1_4096x4096"] = {
        "recipe": "torch.manual_seed(0); (torch.randn(4096, 4096) * 0.02).to(torch.bfloat16)",
        "w_sha256": hashlib.sha256(bits(w).tobytes()).hexdigest(),
        "base": int(base), "n_esc": int(esc[0].numel()),
        "data_sha256": hashlib.sha256(data.numpy().tobytes()).hexdigest(),
        "esc_sha256": hashlib.sha256(np.stack([e.numpy().astype(np.int64) for e in esc]).tobytes()).hexdigest(),
    }
    with open(os.path.join(HERE, "golden_summary.json"), "w") as f:
        json.dump(summary, f, indent=1)
    print(json.dumps(summary, indent=1))


if __name__ == "__main__":
    main()
