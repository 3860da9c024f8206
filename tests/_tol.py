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
