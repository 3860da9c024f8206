"""Tolerance helpers shared by the parity tests.

The reference's own tests compare with absolute tolerances and ``rtol=0``
(1e-4 for Linear/Conv/BN/MHA, 1e-5 for activations). The build's bar is stated
relative to the data: ≤1e-5 on means and ≤1e-4 on variances. Means near zero
make an element-wise relative error ill-posed, so ``rel_err`` measures the
largest element error against the tensor's own scale (max |reference|), which
is the normwise form of that bar.
"""

from __future__ import annotations

import numpy as np
import torch

MEAN_RTOL = 1e-5
VAR_RTOL = 1e-4


def _arr(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().double().numpy()
    return np.asarray(x, dtype=np.float64)


def rel_err(got, ref) -> float:
    g, r = _arr(got), _arr(ref)
    assert g.shape == r.shape, (g.shape, r.shape)
    if g.size == 0:
        return 0.0
    scale = max(np.abs(r).max(), 1e-30)
    return float(np.abs(g - r).max() / scale)


def assert_rel(got, ref, tol, what=""):
    e = rel_err(got, ref)
    assert e <= tol, f"{what}: normwise relative error {e:.3e} > {tol:.1e}"


def var_update_err(S_got, S_ref, S_prev) -> float:
    """Error of updated variances measured against the pre-update variance.

    A variance update that nearly cancels (S' ≈ 5e-5·S) amplifies fp32
    summation-order noise by ~2e4 relative to S'; measuring the difference
    against S (the quantity the update was computed from) keeps the bar
    meaningful. Elements where either side hit the 1e-5 floor are excluded
    and counted by ``floor_flips``.
    """
    g, r, p = _arr(S_got), _arr(S_ref), _arr(S_prev)
    keep = ~((g == np.float32(1e-5)) ^ (r == np.float32(1e-5)))
    if not keep.any():
        return 0.0
    return float((np.abs(g - r)[keep] / np.maximum(np.abs(p[keep]), 1e-30)).max())


def floor_flips(S_got, S_ref) -> int:
    g, r = _arr(S_got), _arr(S_ref)
    return int(((g == np.float32(1e-5)) ^ (r == np.float32(1e-5))).sum())


def assert_as_accurate(got, ref32, exact, factor=2.0, floor=1e-6, what=""):
    """For ill-conditioned closed forms (ReLU variance, Remax): the result's
    normwise error against the float64 evaluation ``exact`` must be within
    ``factor`` times the reference's own float32 error, plus ``floor``."""
    e_got, e_ref = rel_err(got, exact), rel_err(ref32, exact)
    assert e_got <= factor * e_ref + floor, (
        f"{what}: error vs float64 {e_got:.3e} exceeds {factor}x the reference's "
        f"{e_ref:.3e} + {floor:.0e}")


def elem_check(got, ref32, ref64, tol, floor=1e-6):
    """Element-wise relative check of a sign-definite tensor (variances and
    variance deltas) against the float32 reference, with the reference's own
    float32 error as the allowance where that is larger.

    Element i passes if |g − r32| ≤ tol·|r32|, or if |g − r64| ≤ 2·|r32 − r64|
    + tol·|r64|: where the reference's float32 result is itself further than
    the bar from the float64 evaluation (closed forms that cancel: the ReLU
    variance, Remax), the result must be at least as close to float64 as the
    reference is (twice its error). Elements smaller than ``floor``·max|r32| are
    measured against floor·max|r32| (exact zeros of switched-off units).

    Returns (worst, fallbacks, plain): worst ≤ 1 passes (the largest over
    elements of the smaller of the two ratios to their bars), fallbacks counts
    the elements that needed the second branch, plain is the largest
    element-wise relative error against float32.
    """
    g, a, b = _arr(got), _arr(ref32), _arr(ref64)
    assert g.shape == a.shape == b.shape, (g.shape, a.shape, b.shape)
    if g.size == 0:
        return 0.0, 0, 0.0
    fl = floor * max(np.abs(a).max(), 1e-300)
    den32 = np.maximum(np.abs(a), fl)
    den64 = np.maximum(np.abs(b), fl)
    e32 = np.abs(g - a) / den32
    r1 = e32 / tol
    r2 = np.abs(g - b) / (2.0 * np.abs(a - b) + tol * den64)
    r = np.minimum(r1, r2)
    return float(r.max()), int(((r1 > 1) & (r2 <= 1)).sum()), float(e32.max())


def norm_check(got, ref32, ref64, tol):
    """Normwise form of ``elem_check`` for means (which cross zero): passes if
    rel_err(g, r32) ≤ tol, or if rel_err(g, r64) ≤ 2·rel_err(r32, r64) + tol.
    Returns (worst, used_fallback, plain)."""
    e32 = rel_err(got, ref32)
    r1 = e32 / tol
    r2 = rel_err(got, ref64) / (2.0 * rel_err(ref32, ref64) + tol)
    return float(min(r1, r2)), bool(r1 > 1 and r2 <= 1), e32
