"""Shared helpers for the GPU parity tests: seeded inputs (the benchmark's N(0, 0.02) weights, optionally with
1% of them scaled x256; N(0, 1) tokens) and comparison rules."""
import numpy as np
import torch


def bits_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def weight(n, k, seed=0, scale=0.02, escape_frac=0.0, device="cuda"):
    """W = (randn(n, k) * scale) as BF16 (torch seed), optionally with a fraction of weights scaled x256 at
    positions randperm(n*k, seed 2) -- the benchmark's escape variant."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * scale
    if escape_frac:
        idx = torch.randperm(n * k, generator=torch.Generator().manual_seed(2))[: int(n * k * escape_frac)]
        w.view(-1)[idx] *= 256
    return w.to(torch.bfloat16).to(device)


def tokens(m, k, seed=1, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(m, k, generator=g).to(torch.bfloat16).to(device)


def assert_close_bf16(out: torch.Tensor, ref_f32: torch.Tensor, rtol=1e-2, atol=1e-2):
    """The path's tolerance: BF16 outputs within rtol 1e-2 / atol 1e-2 of an FP32-accumulated reference."""
    o = out.float()
    err = (o - ref_f32).abs()
    bound = atol + rtol * ref_f32.abs()
    bad = err > bound
    assert not bool(bad.any()), f"{int(bad.sum())} of {bad.numel()} outside tolerance; max err {float(err.max())}"
    assert bool(torch.isfinite(o).all())


def assert_reference_norms(out: torch.Tensor, ref: torch.Tensor, tol=1e-2):
    """The reference's own random-input acceptance rule (S:297-317): global relative norm <= tol/4 and per-row
    norm <= tol (rows normalised by max(||ref_r||, 0.1 * mean ||ref_r||))."""
    diff = out.double() - ref.double()
    rn = ref.double().norm(dim=1)
    rows = diff.norm(dim=1) / torch.maximum(rn, 0.1 * rn.mean())
    assert float(diff.norm() / ref.double().norm()) <= tol / 4
    assert float(rows.max()) <= tol
