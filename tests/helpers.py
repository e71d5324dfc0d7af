"""Shared test helpers: golden fixtures and tolerance checks."""
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerance of the reference's fp32 formulation, as stated by the north star.
RTOL = 1e-4
ATOL = 1e-5


def golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: torch.from_numpy(np.array(z[k])) for k in z.files}


def scaled_atol(expected, atol=ATOL):
    """The absolute tolerance applies at unit scale: for a tensor whose
    entries reach S > 1 it is atol * S.  Entries of the parameter gradients are
    sums over tokens of terms of size ~S; near-zero entries carry fp32 rounding
    error ~eps32 * S * sqrt(tokens), which an unscaled 1e-5 cannot absorb -- the
    reference's own fp32 formulation misses the unscaled bound by up to 10x on
    phi gradients with alpha = 1."""
    return atol * max(1.0, expected.detach().abs().max().item() if expected.numel() else 1.0)


def close(actual, expected, rtol=RTOL, atol=ATOL, what="", scaled=False):
    """|actual - expected| <= atol + rtol |expected| elementwise.  `scaled`
    widens atol to the tensor's scale (scaled_atol) and is meant only for the
    batch-reduced parameter gradients; per-token outputs (out, grad_x, ...)
    are held to the unscaled bound.  Returns the max abs error (also printed)."""
    a = actual.detach().double().cpu()
    e = expected.detach().double().cpu()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} != {tuple(e.shape)}"
    err = (a - e).abs()
    if scaled:
        atol = scaled_atol(e, atol)
    bound = atol + rtol * e.abs()
    bad = err > bound
    max_err = err.max().item() if err.numel() else 0.0
    print(f"{what}: max_abs_err={max_err:.3g} (atol={atol:.3g}, rtol={rtol:g})")
    if bad.any():
        idx = int(torch.argmax((err - bound).reshape(-1)))
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{a.numel()} elements outside rtol={rtol} atol={atol}; "
            f"worst at flat index {idx}: actual={a.reshape(-1)[idx].item():.8g} "
            f"expected={e.reshape(-1)[idx].item():.8g} max_abs_err={max_err:.3g}")
    return max_err


def close_param(actual, expected, rtol=RTOL, atol=ATOL, what=""):
    """Parameter gradients (sums over the batch): atol at the tensor's scale."""
    return close(actual, expected, rtol, atol, what, scaled=True)


def rel_err(actual, expected):
    a = actual.detach().double().cpu()
    e = expected.detach().double().cpu()
    return ((a - e).norm() / e.norm().clamp_min(1e-30)).item()


def close_ref(actual, ref32, truth, rtol=RTOL, atol=ATOL, what="", scaled=False):
    """Parity with the reference's fp32 result `ref32`, judged against exact
    arithmetic `truth` (the same formulation evaluated in fp64):

    * |actual - truth| <= atol + rtol |truth|   (the stated tolerance), and
    * |actual - ref32| <= atol + rtol |ref32| + |ref32 - truth|, i.e. the
      tolerance widened by the reference's own fp32 rounding error -- the fp32
      reference itself misses exact arithmetic by up to 3.6x the tolerance on
      ill-conditioned gradients (b_res, b_pre at BASELINE cfg1).

    `scaled` (parameter gradients only) applies atol at the tensor's scale.
    """
    close(actual, truth, rtol, atol, what + " (vs fp64 truth)", scaled=scaled)
    a = actual.detach().double().cpu()
    r = ref32.detach().double().cpu()
    t = truth.detach().double().cpu()
    bound = (scaled_atol(t, atol) if scaled else atol) + rtol * r.abs() + (r - t).abs()
    bad = (a - r).abs() > bound
    assert not bad.any(), f"{what}: {int(bad.sum())} elements outside the widened bound vs fp32 reference"
