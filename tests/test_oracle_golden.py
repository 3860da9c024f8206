"""Pin the CPU oracle to the reference: every oracle function against the golden
vectors produced by running triton-tagi itself (tests/golden/make_golden.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle.moments as F
import oracle.net as ON
from _nets import build, golden_params, load, params
from _tol import MEAN_RTOL, VAR_RTOL, assert_as_accurate, assert_rel, rel_err, var_update_err

T = torch.from_numpy


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_gemm_family(golden, tag):
    z = golden("kernels")
    g = {k: T(z[f"gemm_{tag}_{k}"]) for k in ("ma", "Sa", "mw", "Sw", "Sb", "dmz", "dSz")}
    assert_rel(F.var_forward(g["ma"], g["Sa"], g["mw"], g["Sw"], g["Sb"]), z[f"gemm_{tag}_Sz"],
               VAR_RTOL, "var_forward")
    d_ma, d_Sa = F.backward_delta(g["dmz"], g["dSz"], g["mw"])
    assert_rel(d_ma, z[f"gemm_{tag}_d_ma"], MEAN_RTOL, "d_ma")
    assert_rel(d_Sa, z[f"gemm_{tag}_d_Sa"], VAR_RTOL, "d_Sa")
    gmw, gSw = F.weight_grad(g["ma"], g["dmz"], g["dSz"])
    assert_rel(gmw, z[f"gemm_{tag}_gmw"], MEAN_RTOL, "gmw")
    assert_rel(gSw, z[f"gemm_{tag}_gSw"], VAR_RTOL, "gSw")


@pytest.mark.parametrize("cap", [0.1, 2.0, 3.0])
def test_capped_update(golden, cap):
    z = golden("kernels")
    m, S = F.capped_update(T(z["upd_m"]), T(z["upd_S"]), T(z["upd_dm"]), T(z["upd_dS"]), cap)
    # Element-wise float arithmetic: agree to within one rounding of the cap
    # division (the interpreter and IEEE division can differ by 1 ulp).
    np.testing.assert_allclose(m.numpy(), z[f"upd_cap{cap}_m"], rtol=2.5e-7, atol=0)
    np.testing.assert_allclose(S.numpy(), z[f"upd_cap{cap}_S"], rtol=2.5e-7, atol=0)


def test_cap_factor():
    assert [F.get_cap_factor(b) for b in (1, 2, 255, 256, 1024)] == [0.1, 2.0, 2.0, 3.0, 3.0]


def test_innovation(golden):
    z = golden("kernels")
    dm, dv = F.innovation(T(z["inn_y"]), T(z["inn_mu"]), T(z["inn_var"]), 0.05)
    np.testing.assert_allclose(dm.numpy(), z["inn_dmu"], rtol=1e-6, atol=0)
    np.testing.assert_allclose(dv.numpy(), z["inn_dvar"], rtol=1e-6, atol=0)


def test_relu(golden):
    z = golden("kernels")
    mz, Sz = T(z["relu_mz"]), T(z["relu_Sz"])
    ma, Sa, J = F.relu_moments(mz, Sz)
    ex = F.relu_moments(mz.double(), Sz.double())
    for got, key, exact in zip((ma, Sa, J), ("relu_ma", "relu_Sa", "relu_J"), ex):
        assert_as_accurate(got, z[key], exact, floor=1e-6, what=key)


@pytest.mark.parametrize("tag", ["k10", "k64", "k512"])
def test_remax(golden, tag):
    z = golden("kernels")
    mz, Sz = T(z[f"remax_{tag}_mz"]), T(z[f"remax_{tag}_Sz"])
    got = F.remax(mz, Sz)
    ex = F.remax(mz.double(), Sz.double())
    for g, nm, x in zip(got, ("ma", "Sa", "J"), ex):
        assert_as_accurate(g, z[f"remax_{tag}_{nm}"], x, floor=1e-6, what=f"remax {nm}")


def test_attention_products(golden):
    z = golden("kernels")
    ma, va, mb, vb = (T(z[k]) for k in ("att_ma", "att_va", "att_mb", "att_vb"))
    tr = lambda t: t.transpose(-1, -2)  # noqa: E731
    assert_rel(F.bmm_tagi_var(ma, va, tr(mb), tr(vb), 0.25), z["att_var_t"], VAR_RTOL, "var")
    m, v = F.bmm_shared_right(ma, va, tr(mb), 0.5)
    assert_rel(m, z["att_right_m"], MEAN_RTOL, "right m")
    assert_rel(v, z["att_right_v"], VAR_RTOL, "right v")
    m, v = F.bmm_shared_left(ma, T(z["att_bm"]), T(z["att_bv"]), 0.5)
    assert_rel(m, z["att_left_m"], MEAN_RTOL, "left m")
    assert_rel(v, z["att_left_v"], VAR_RTOL, "left v")


@pytest.mark.parametrize("tag,k,s,p", [("k3s1p1", 3, 1, 1), ("k3s2p1", 3, 2, 1),
                                       ("k2s2p0", 2, 2, 0), ("k5s1p2", 5, 1, 2)])
def test_im2col_col2im(golden, tag, k, s, p):
    z = golden("kernels")
    x = T(z["im2col_x"])
    cols = F.im2col(x, k, s, p)
    np.testing.assert_array_equal(cols.numpy(), z[f"im2col_{tag}"])
    img = F.col2im(cols * 0.5 + 1.0, 2, 3, 9, 7, k, s, p)
    np.testing.assert_allclose(img.numpy(), z[f"col2im_{tag}"], rtol=1e-6, atol=1e-5)
    fold = F.col2im(cols * 0.5 + 1.0, 2, 3, 9, 7, k, s, p, adjoint=True)
    if s == 1:  # the reference's gather is the adjoint at stride 1 ...
        np.testing.assert_allclose(fold.numpy(), img.numpy(), rtol=1e-6, atol=1e-5)
    else:       # ... and gathers extra taps at stride > 1 (conv2d.py:126)
        assert np.abs(fold.numpy() - img.numpy()).max() > 0.1


@pytest.mark.parametrize("name", ["mlp", "cnn", "res", "tfm"])
def test_trajectory(golden, name):
    """Short Sequential.step trajectories from identical initial parameters."""
    z = golden(f"traj_{name}")
    layers = build(name, ON)
    load(layers, golden_params(z, 0))
    net = ON.Sequential(layers)
    x, y = T(z["x"]), T(z["y"])
    steps = int(z["steps"])
    for s in range(steps):
        mu, var = net.step(x, y, 0.05)
        assert_rel(mu, z[f"mu_{s}"], 1e-4, f"step {s} mu")
        assert_rel(var, z[f"var_{s}"], 1e-3, f"step {s} var")
    got = params(layers)
    ref = golden_params(z, steps)
    prev = golden_params(z, 0)
    for i, (g, r) in enumerate(zip(got, ref)):
        if i % 2 == 0:
            assert rel_err(g, r) <= 1e-4, f"param {i}: {rel_err(g, r):.3e}"
        else:
            assert var_update_err(g, r, prev[i]) <= 1e-3, f"param {i}"
