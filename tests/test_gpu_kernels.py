"""Kernel parity on the GPU: every libtagi_b200 entry point against the CPU
oracle (float64 where the bar is relative error) and against the golden
vectors that the reference itself produced."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle.moments as F
from _tol import MEAN_RTOL, VAR_RTOL, assert_as_accurate, assert_rel

pytestmark = pytest.mark.gpu
DEV = "cuda"


def g(t):
    return torch.as_tensor(t).to(DEV, torch.float32)


def d64(t):
    return torch.as_tensor(t).detach().cpu().double()


def rnd(gen, *shape, kind="n", scale=1.0, lo=0.0):
    if kind == "n":
        return torch.randn(*shape, generator=gen) * scale
    return torch.rand(*shape, generator=gen) * scale + lo


SHAPES = [(37, 27, 10), (256, 784, 256), (513, 300, 130), (8, 4608, 64), (4096, 64, 1)]


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_var_forward_and_linear_forward(M, K, N):
    from triton_tagi.kernels.common import triton_fused_var_forward
    from triton_tagi import Linear

    gen = torch.Generator().manual_seed(M * 7 + K)
    ma, Sa = rnd(gen, M, K), rnd(gen, M, K, kind="u", scale=1e-2, lo=1e-4)
    mw, Sw = rnd(gen, K, N, scale=K**-0.5), rnd(gen, K, N, kind="u", scale=1.0 / K)
    mb, Sb = rnd(gen, 1, N, scale=0.1), rnd(gen, 1, N, kind="u", scale=1e-3)
    ref_S = F.var_forward(d64(ma), d64(Sa), d64(mw), d64(Sw), d64(Sb))
    assert_rel(triton_fused_var_forward(g(ma), g(Sa), g(mw), g(Sw), g(Sb)), ref_S, VAR_RTOL, "Sz")
    lin = Linear(K, N, device=DEV)
    lin.mw, lin.Sw, lin.mb, lin.Sb = g(mw), g(Sw), g(mb), g(Sb)
    mz, Sz = lin.forward(g(ma), g(Sa))
    assert_rel(mz, F.mean_forward(d64(ma), d64(mw), d64(mb)), MEAN_RTOL, "mz")
    assert_rel(Sz, ref_S, VAR_RTOL, "Sz (linear)")


def test_var_forward_strided_views():
    from triton_tagi.kernels.common import triton_fused_var_forward

    gen = torch.Generator().manual_seed(3)
    ma, Sa = rnd(gen, 40, 33).T, rnd(gen, 40, 33, kind="u").T   # (33, 40), column-major
    mw, Sw = rnd(gen, 17, 40).T, rnd(gen, 17, 40, kind="u").T   # (40, 17), column-major
    Sb = rnd(gen, 1, 17, kind="u")
    got = triton_fused_var_forward(g(ma.T).T, g(Sa.T).T, g(mw.T).T, g(Sw.T).T, g(Sb))
    assert_rel(got, F.var_forward(d64(ma), d64(Sa), d64(mw), d64(Sw), d64(Sb)), VAR_RTOL, "Sz")


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_backward_delta_and_weight_grad(M, K, N):
    from triton_tagi.kernels.common import triton_fused_backward_delta, triton_fused_weight_grad

    gen = torch.Generator().manual_seed(M + 11 * N)
    a = rnd(gen, M, K)
    mw = rnd(gen, K, N, scale=K**-0.5)
    dmz, dSz = rnd(gen, M, N, scale=0.1), -rnd(gen, M, N, kind="u", scale=1e-2)
    d_ma, d_Sa = triton_fused_backward_delta(g(dmz), g(dSz), g(mw))
    r_ma, r_Sa = F.backward_delta(d64(dmz), d64(dSz), d64(mw))
    assert_rel(d_ma, r_ma, MEAN_RTOL, "d_ma")
    assert_rel(d_Sa, r_Sa, VAR_RTOL, "d_Sa")
    gm, gS = triton_fused_weight_grad(g(a), g(dmz), g(dSz))
    rm, rS = F.weight_grad(d64(a), d64(dmz), d64(dSz))
    assert_rel(gm, rm, MEAN_RTOL, "grad_mw")
    assert_rel(gS, rS, VAR_RTOL, "grad_Sw")


def test_weight_grad_split_reduction_is_deterministic():
    from triton_tagi.kernels.common import triton_fused_weight_grad

    gen = torch.Generator().manual_seed(5)
    a, dmz, dSz = rnd(gen, 50000, 27), rnd(gen, 50000, 10), rnd(gen, 50000, 10, kind="u")
    r1 = triton_fused_weight_grad(g(a), g(dmz), g(dSz))
    r2 = triton_fused_weight_grad(g(a), g(dmz), g(dSz))
    assert torch.equal(r1[0], r2[0]) and torch.equal(r1[1], r2[1])
    rm, rS = F.weight_grad(d64(a), d64(dmz), d64(dSz))
    assert_rel(r1[0], rm, MEAN_RTOL, "gmw")
    assert_rel(r1[1], rS, VAR_RTOL, "gSw")


def test_golden_gemm_family(golden):
    from triton_tagi.kernels.common import (triton_fused_backward_delta, triton_fused_var_forward,
                                            triton_fused_weight_grad)

    z = golden("kernels")
    for tag in ("a", "b", "c"):
        t = {k: g(z[f"gemm_{tag}_{k}"]) for k in ("ma", "Sa", "mw", "Sw", "Sb", "dmz", "dSz")}
        assert_rel(triton_fused_var_forward(t["ma"], t["Sa"], t["mw"], t["Sw"], t["Sb"]),
                   z[f"gemm_{tag}_Sz"], VAR_RTOL, "Sz")
        d_ma, d_Sa = triton_fused_backward_delta(t["dmz"], t["dSz"], t["mw"])
        assert_rel(d_ma, z[f"gemm_{tag}_d_ma"], MEAN_RTOL, "d_ma")
        assert_rel(d_Sa, z[f"gemm_{tag}_d_Sa"], VAR_RTOL, "d_Sa")
        gm, gS = triton_fused_weight_grad(t["ma"], t["dmz"], t["dSz"])
        assert_rel(gm, z[f"gemm_{tag}_gmw"], MEAN_RTOL, "gmw")
        assert_rel(gS, z[f"gemm_{tag}_gSw"], VAR_RTOL, "gSw")


@pytest.mark.parametrize("cap", [0.1, 2.0, 3.0])
def test_capped_update_golden(golden, cap):
    from triton_tagi.update.parameters import update_parameters

    z = golden("kernels")
    m, S = g(z["upd_m"]), g(z["upd_S"])
    update_parameters(m, S, g(z["upd_dm"]), g(z["upd_dS"]), cap)
    np.testing.assert_allclose(m.cpu().numpy(), z[f"upd_cap{cap}_m"], rtol=2.5e-7, atol=0)
    np.testing.assert_allclose(S.cpu().numpy(), z[f"upd_cap{cap}_S"], rtol=2.5e-7, atol=0)
    # odd length and offset view take the scalar path
    m2, S2 = g(z["upd_m"])[1:], g(z["upd_S"])[1:]
    update_parameters(m2, S2, g(z["upd_dm"])[1:], g(z["upd_dS"])[1:], cap)
    np.testing.assert_allclose(m2.cpu().numpy(), z[f"upd_cap{cap}_m"][1:], rtol=2.5e-7, atol=0)


def test_innovation_golden(golden):
    from triton_tagi.update.observation import compute_innovation

    z = golden("kernels")
    dm, dv = compute_innovation(g(z["inn_y"]), g(z["inn_mu"]), g(z["inn_var"]), 0.05)
    np.testing.assert_allclose(dm.cpu().numpy(), z["inn_dmu"], rtol=1e-6, atol=0)
    np.testing.assert_allclose(dv.cpu().numpy(), z["inn_dvar"], rtol=1e-6, atol=0)


def test_relu_golden(golden):
    from triton_tagi.layers.relu import bayesian_relu

    z = golden("kernels")
    mz, Sz = torch.from_numpy(z["relu_mz"]), torch.from_numpy(z["relu_Sz"])
    got = bayesian_relu(g(mz), g(Sz))
    ex = F.relu_moments(mz.double(), Sz.double())
    for t, key, x in zip(got, ("relu_ma", "relu_Sa", "relu_J"), ex):
        assert_as_accurate(t.cpu(), z[key], x, floor=1e-6, what=key)
    odd = bayesian_relu(g(mz[:4093]), g(Sz[:4093]))  # scalar path
    assert torch.equal(odd[0].cpu(), got[0][:4093].cpu())


@pytest.mark.parametrize("tag", ["k10", "k64", "k512"])
def test_remax_golden(golden, tag):
    from triton_tagi.layers.remax import triton_remax

    z = golden("kernels")
    mz, Sz = torch.from_numpy(z[f"remax_{tag}_mz"]), torch.from_numpy(z[f"remax_{tag}_Sz"])
    got = triton_remax(g(mz), g(Sz))
    ex = F.remax(mz.double(), Sz.double())
    # var_a = (exp(v)-1)·μ² and cov(A,M) = (exp(c)-1)·… cancel for small v, c:
    # a 1-ulp difference between two exp implementations becomes ~1e-4 relative,
    # so the bar is 4x the reference's own float32 error (same formula).
    for t, nm, x in zip(got, ("ma", "Sa", "J"), ex):
        assert_as_accurate(t.cpu(), z[f"remax_{tag}_{nm}"], x, factor=4.0, floor=1e-6,
                           what=f"remax {nm}")


@pytest.mark.parametrize("K", [3, 33, 200, 512, 700, 1100])
def test_remax_sizes(K):
    """Rows of every Remax kernel (registers up to 128 classes, shared memory up
    to 1024, global recomputation beyond)."""
    from triton_tagi.layers.remax import triton_remax

    gen = torch.Generator().manual_seed(K)
    mz, Sz = rnd(gen, 65, K, scale=2.0), rnd(gen, 65, K, kind="u", scale=2.0, lo=1e-3)
    got = triton_remax(g(mz), g(Sz))
    ref32 = F.remax(mz, Sz)
    ex = F.remax(mz.double(), Sz.double())
    for t, r, x, nm in zip(got, ref32, ex, ("ma", "Sa", "J")):
        assert_as_accurate(t.cpu(), r, x, factor=4.0, floor=1e-6, what=nm)


def test_attention_products_golden(golden):
    from triton_tagi.kernels.attention import bmm_shared_left, bmm_shared_right, bmm_tagi_var

    z = golden("kernels")
    ma, va, mb, vb = (g(z[k]) for k in ("att_ma", "att_va", "att_mb", "att_vb"))
    tr = lambda t: t.transpose(-1, -2)  # noqa: E731
    assert_rel(bmm_tagi_var(ma, va, tr(mb), tr(vb), 0.25), z["att_var_t"], VAR_RTOL, "var")
    m, v = bmm_shared_right(ma, va, tr(mb), 0.5)
    assert_rel(m, z["att_right_m"], MEAN_RTOL, "right m")
    assert_rel(v, z["att_right_v"], VAR_RTOL, "right v")
    m, v = bmm_shared_left(ma, g(z["att_bm"]), g(z["att_bv"]), 0.5)
    assert_rel(m, z["att_left_m"], MEAN_RTOL, "left m")
    assert_rel(v, z["att_left_v"], VAR_RTOL, "left v")
    with pytest.raises(ValueError):
        bmm_tagi_var(ma, va, mb, vb)


def test_attention_products_fused_mean():
    from triton_tagi.kernels.attention import bmm_tagi_moments

    gen = torch.Generator().manual_seed(9)
    ma, va = rnd(gen, 4, 8, 64, 32), rnd(gen, 4, 8, 64, 32, kind="u")
    mb, vb = rnd(gen, 4, 8, 32, 48), rnd(gen, 4, 8, 32, 48, kind="u")
    m, v = bmm_tagi_moments(g(ma), g(va), g(mb), g(vb), 0.125, 0.125**2)
    assert_rel(m, 0.125 * (d64(ma) @ d64(mb)), MEAN_RTOL, "mean")
    assert_rel(v, F.bmm_tagi_var(d64(ma), d64(va), d64(mb), d64(vb), 0.125**2), VAR_RTOL, "var")


@pytest.mark.parametrize("tag,k,s,p", [("k3s1p1", 3, 1, 1), ("k3s2p1", 3, 2, 1),
                                       ("k2s2p0", 2, 2, 0), ("k5s1p2", 5, 1, 2)])
def test_im2col_col2im_golden(golden, tag, k, s, p):
    from triton_tagi._lib import lib, stream

    z = golden("kernels")
    x = g(z["im2col_x"])
    N, C, H, W = x.shape
    Ho, Wo = F.conv_out_hw(H, W, k, s, p, 1)
    pm = torch.empty(N * Ho * Wo, C * k * k, device=DEV)
    pS = torch.empty_like(pm)
    lib()("tagi_im2col", x.data_ptr(), x.data_ptr(), pm.data_ptr(), pS.data_ptr(), N, C, H, W, k,
          s, p, 1, stream(x))
    np.testing.assert_array_equal(pm.cpu().numpy(), z[f"im2col_{tag}"])
    cols = pm * 0.5 + 1.0
    for mode, adjoint in ((0, False), (1, True)):
        out = torch.empty(N, C, H, W, device=DEV)
        out2 = torch.empty_like(out)
        lib()("tagi_col2im", cols.data_ptr(), cols.data_ptr(), out.data_ptr(), out2.data_ptr(), N,
              C, H, W, k, s, p, 1, mode, stream(x))
        ref = F.col2im(cols.cpu(), N, C, H, W, k, s, p, 1, adjoint=adjoint)
        np.testing.assert_allclose(out.cpu().numpy(), ref.numpy(), rtol=1e-6, atol=1e-5)
        if mode == 0:  # the reference's own gather
            np.testing.assert_allclose(out.cpu().numpy(), z[f"col2im_{tag}"], rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("N,C,H,k,p,pt", [(4, 64, 32, 3, 1, 2), (4, 128, 16, 3, 1, 2),
                                          (8, 256, 8, 3, 1, 2), (4, 64, 32, 2, 0, 1),
                                          (3, 12, 20, 3, 1, 1), (2, 8, 12, 3, 1, 2)])
def test_col2im_stride2_staged(N, C, H, k, p, pt):
    """Stride-2 gathers of the ResNet downsampling layers (16-byte staged
    kernel: C and W multiples of 4), both modes, against the oracle's gather
    (same taps, same order)."""
    from triton_tagi._lib import lib, stream

    Ho, Wo = F.conv_out_hw(H, H, k, 2, p, pt)
    gen = torch.Generator().manual_seed(C + H + k)
    cm = rnd(gen, N * Ho * Wo, C * k * k)
    cS = rnd(gen, N * Ho * Wo, C * k * k, kind="u")
    dm, dS = g(cm), g(cS)
    for mode, adjoint in ((0, False), (1, True)):
        om = torch.empty(N, C, H, H, device=DEV)
        oS = torch.empty_like(om)
        lib()("tagi_col2im", dm.data_ptr(), dS.data_ptr(), om.data_ptr(), oS.data_ptr(),
              N, C, H, H, k, 2, p, pt, mode, stream(om))
        for got, src in ((om, cm), (oS, cS)):
            ref = F.col2im(src, N, C, H, H, k, 2, p, pt, adjoint=adjoint)
            np.testing.assert_allclose(got.cpu().numpy(), ref.numpy(), rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("C,k,s,p,pt", [(4, 3, 1, 1, 1), (8, 3, 2, 1, 1), (4, 2, 2, 0, 1),
                                       (12, 5, 1, 2, 2), (16, 1, 1, 0, 1)])
def test_im2col_vectorised_rows(C, k, s, p, pt):
    """Patch rows with C*k*k a multiple of 4 (16-byte stores), mean and variance
    together and the mean alone, bit-exact against the oracle's unfold."""
    from triton_tagi._lib import lib, stream

    gen = torch.Generator().manual_seed(C * 10 + k)
    N, H, W = 3, 11, 10
    xm, xS = rnd(gen, N, C, H, W), rnd(gen, N, C, H, W, kind="u")
    Ho, Wo = F.conv_out_hw(H, W, k, s, p, pt)
    dm, dS = g(xm), g(xS)  # device copies held for the calls
    pm = torch.empty(N * Ho * Wo, C * k * k, device=DEV)
    pS = torch.empty_like(pm)
    lib()("tagi_im2col", dm.data_ptr(), dS.data_ptr(), pm.data_ptr(), pS.data_ptr(), N, C, H, W,
          k, s, p, pt, stream(pm))
    np.testing.assert_array_equal(pm.cpu().numpy(), F.im2col(xm, k, s, p, pt).numpy())
    np.testing.assert_array_equal(pS.cpu().numpy(), F.im2col(xS, k, s, p, pt).numpy())
    only = torch.full_like(pm, 7.0)
    lib()("tagi_im2col", dm.data_ptr(), None, only.data_ptr(), None, N, C, H, W, k, s, p, pt,
          stream(pm))
    np.testing.assert_array_equal(only.cpu().numpy(), F.im2col(xm, k, s, p, pt).numpy())


@pytest.mark.parametrize("C,H,k,s,p,pt", [(128, 16, 3, 1, 1, 1), (64, 32, 3, 2, 1, 2),
                                          (64, 32, 2, 2, 0, 1), (512, 4, 3, 1, 1, 1),
                                          (12, 20, 3, 2, 1, 1), (6, 8, 2, 1, 0, 1)])
def test_im2col_row_staged(C, H, k, s, p, pt):
    """ResNet shapes (W and C*k*k multiples of 4: every channel's input lines
    staged at once, 16-byte stores), both planes and the mean alone, bit-exact
    against the oracle's unfold."""
    from triton_tagi._lib import lib, stream

    gen = torch.Generator().manual_seed(C + H + k)
    N = 3
    xm, xS = rnd(gen, N, C, H, H), rnd(gen, N, C, H, H, kind="u")
    Ho, Wo = F.conv_out_hw(H, H, k, s, p, pt)
    dm, dS = g(xm), g(xS)
    pm = torch.empty(N * Ho * Wo, C * k * k, device=DEV)
    pS = torch.empty_like(pm)
    lib()("tagi_im2col", dm.data_ptr(), dS.data_ptr(), pm.data_ptr(), pS.data_ptr(), N, C, H, H,
          k, s, p, pt, stream(pm))
    np.testing.assert_array_equal(pm.cpu().numpy(), F.im2col(xm, k, s, p, pt).numpy())
    np.testing.assert_array_equal(pS.cpu().numpy(), F.im2col(xS, k, s, p, pt).numpy())
    only = torch.full_like(pm, 7.0)
    lib()("tagi_im2col", dm.data_ptr(), None, only.data_ptr(), None, N, C, H, H, k, s, p, pt,
          stream(pm))
    np.testing.assert_array_equal(only.cpu().numpy(), F.im2col(xm, k, s, p, pt).numpy())


@pytest.mark.parametrize("C,H,W,k,s,p,pt", [(24, 6, 300, 3, 1, 1, 1), (10, 5, 700, 5, 2, 2, 2),
                                             (64, 9, 9, 3, 1, 1, 1), (3, 33, 31, 7, 2, 3, 1)])
def test_im2col_channel_slices(C, H, W, k, s, p, pt):
    """Wide images whose staged input lines exceed the kernel's shared-memory
    budget (several channel slices per patch row), and slices of more or fewer
    patch columns than threads; bit-exact against the oracle's unfold."""
    from triton_tagi._lib import lib, stream

    gen = torch.Generator().manual_seed(C + W)
    N = 2
    xm, xS = rnd(gen, N, C, H, W), rnd(gen, N, C, H, W, kind="u")
    Ho, Wo = F.conv_out_hw(H, W, k, s, p, pt)
    dm, dS = g(xm), g(xS)
    pm = torch.empty(N * Ho * Wo, C * k * k, device=DEV)
    pS = torch.empty_like(pm)
    lib()("tagi_im2col", dm.data_ptr(), dS.data_ptr(), pm.data_ptr(), pS.data_ptr(), N, C, H, W,
          k, s, p, pt, stream(pm))
    np.testing.assert_array_equal(pm.cpu().numpy(), F.im2col(xm, k, s, p, pt).numpy())
    np.testing.assert_array_equal(pS.cpu().numpy(), F.im2col(xS, k, s, p, pt).numpy())
    only = torch.full_like(pm, 7.0)
    lib()("tagi_im2col", dm.data_ptr(), None, only.data_ptr(), None, N, C, H, W, k, s, p, pt,
          stream(pm))
    np.testing.assert_array_equal(only.cpu().numpy(), F.im2col(xm, k, s, p, pt).numpy())


@pytest.mark.parametrize("N,C,HW", [(3, 6, 7), (4, 64, 1024), (2, 36, 49), (5, 520, 16),
                                    (3, 12, 20), (1, 100, 4), (2, 8, 1)])
def test_nchw_to_nhwc(N, C, HW):
    """Channels-last copies, one plane and two: the 128-bit tile kernel (C and
    HW multiples of 4) and the general one; exact."""
    from triton_tagi._lib import lib, stream

    gen = torch.Generator().manual_seed(N * C + HW)
    a, b = g(rnd(gen, N, C, HW)), g(rnd(gen, N, C, HW))
    ya, yb = torch.full((N, HW, C), 7.0, device=DEV), torch.full((N, HW, C), 7.0, device=DEV)
    lib()("tagi_nchw_to_nhwc", a.data_ptr(), b.data_ptr(), ya.data_ptr(), yb.data_ptr(), N, C, HW,
          stream(a))
    assert torch.equal(ya, a.permute(0, 2, 1)) and torch.equal(yb, b.permute(0, 2, 1))
    only = torch.full((N, HW, C), 7.0, device=DEV)
    lib()("tagi_nchw_to_nhwc", b.data_ptr(), None, only.data_ptr(), None, N, C, HW, stream(a))
    assert torch.equal(only, b.permute(0, 2, 1))


@pytest.mark.parametrize("C,H,W,k,s,p,pt", [(3, 11, 10, 3, 1, 1, 1), (5, 40, 36, 3, 2, 1, 2),
                                             (4, 9, 700, 5, 1, 2, 1), (2, 5, 2100, 3, 1, 1, 1),
                                             (6, 12, 12, 1, 1, 0, 1), (3, 30, 33, 7, 2, 3, 2),
                                             (4, 16, 21, 3, 1, 1, 2), (2, 7, 10, 5, 1, 1, 1),
                                             (3, 6, 1500, 3, 1, 1, 1), (2, 9, 14, 3, 1, 0, 1)])
def test_im2col_transposed(C, H, W, k, s, p, pt):
    """tagi_im2col_t: the stride-1 kernel (k = 1, 3, 5, zero-padded rows, one or
    several bands), the general band kernel (128-bit stores or not) and the
    element-per-thread kernel of images too wide to stage; bit-exact against the
    transposed unfold."""
    from triton_tagi._lib import lib, stream

    gen = torch.Generator().manual_seed(C * W + k)
    N = 3
    x = rnd(gen, N, C, H, W)
    Ho, Wo = F.conv_out_hw(H, W, k, s, p, pt)
    dx = g(x)
    out = torch.full((C * k * k, N * Ho * Wo), 7.0, device=DEV)
    lib()("tagi_im2col_t", dx.data_ptr(), out.data_ptr(), N, C, H, W, k, s, p, pt, stream(dx))
    np.testing.assert_array_equal(out.cpu().numpy(), F.im2col(x, k, s, p, pt).t().numpy())


@pytest.mark.parametrize("shape,k,s,p,pt", [((2, 3, 9, 7), 3, 2, 1, 2), ((3, 4, 8, 8), 3, 1, 1, 1),
                                            ((2, 5, 16, 16), 2, 2, 0, 1),
                                            ((2, 3, 12, 12), 5, 1, 2, 1)])
def test_conv_layer_against_oracle(shape, k, s, p, pt):
    import oracle.net as ON
    from triton_tagi import Conv2D

    gen = torch.Generator().manual_seed(sum(shape) + k)
    N, C, H, W = shape
    Co = 6
    ma, Sa = rnd(gen, *shape), rnd(gen, *shape, kind="u", scale=0.1)
    torch.manual_seed(0)
    ref = ON.Conv2D(C, Co, k, s, p, pt)
    dev = Conv2D(C, Co, k, s, p, pt, device=DEV)
    for n in ("mw", "Sw", "mb", "Sb"):
        setattr(dev, n, g(getattr(ref, n)))
    rm, rS = ref.forward(ma, Sa)
    gm, gS = dev.forward(g(ma), g(Sa))
    ex_m, ex_S, _ = F.conv_forward(ma.double(), Sa.double(), d64(ref.mw), d64(ref.Sw),
                                   d64(ref.mb), d64(ref.Sb), k, s, p, pt)
    assert_rel(gm, ex_m, MEAN_RTOL, "conv mz")
    assert_rel(gS, ex_S, VAR_RTOL, "conv Sz")
    dmz, dSz = rnd(gen, *rm.shape, scale=0.1), -rnd(gen, *rm.shape, kind="u", scale=0.01)
    for mode in ("reference", "adjoint"):
        dev.col2im_mode = mode
        ref.col2im_adjoint = mode == "adjoint"
        ref.forward(ma, Sa)
        dev.forward(g(ma), g(Sa))
        r_dm, r_dS = ref.backward(dmz, dSz)
        d_dm, d_dS = dev.backward(g(dmz), g(dSz))
        assert_rel(d_dm, r_dm, 1e-5, f"conv d_ma {mode}")
        assert_rel(d_dS, r_dS, 1e-4, f"conv d_Sa {mode}")
        for n in ("delta_mw", "delta_mb"):
            assert_rel(getattr(dev, n), getattr(ref, n), 1e-5, n)
        for n in ("delta_Sw", "delta_Sb"):
            assert_rel(getattr(dev, n), getattr(ref, n), 1e-4, n)


@pytest.mark.parametrize("N,C,H,W", [(8, 16, 6, 6), (3, 5, 7, 5), (1, 600, 2, 2), (64, 4, 16, 16),
                                     (8, 512, 4, 4)])
def test_batchnorm_layer_against_oracle(N, C, H, W):
    """Covers 16-byte and element-wise channel slabs, clusters of 2 to 8 blocks per
    channel, one block per channel (512 or more channels, or one image: a launch
    without clusters), and fewer images than blocks in a cluster."""
    import oracle.net as ON
    from triton_tagi import BatchNorm2D

    gen = torch.Generator().manual_seed(21 + N + C)
    ref, dev = ON.BatchNorm2D(C), BatchNorm2D(C, device=DEV)
    for step in range(2):  # first call initialises running stats, second uses the EMA
        mz, Sz = rnd(gen, N, C, H, W) + 0.3, rnd(gen, N, C, H, W, kind="u", scale=0.2)
        rm, rS = ref.forward(mz, Sz)
        gm, gS = dev.forward(g(mz), g(Sz))
        assert_rel(gm, rm, 1e-5, f"bn ma {step}")
        assert_rel(gS, rS, 1e-4, f"bn Sa {step}")
        assert_rel(dev.running_mean, ref.running_mean, 1e-5, "running_mean")
        assert_rel(dev.running_var, ref.running_var, 1e-5, "running_var")
        assert_rel(dev.mw, ref.mw, 1e-6, "gamma (preserve_var)")
        dm, dS = rnd(gen, N, C, H, W, scale=0.1), -rnd(gen, N, C, H, W, kind="u", scale=0.01)
        r = ref.backward(dm, dS)
        d = dev.backward(g(dm), g(dS))
        assert_rel(d[0], r[0], 1e-5, "bn dmz")
        assert_rel(d[1], r[1], 1e-4, "bn dSz")
        for n, tol in (("delta_mw", 1e-5), ("delta_Sw", 1e-4), ("delta_mb", 1e-5),
                       ("delta_Sb", 1e-4)):
            assert_rel(getattr(dev, n), getattr(ref, n), tol, n)


def test_avgpool_and_add():
    from triton_tagi import AvgPool2D
    from triton_tagi.layers.resblock import triton_add_shortcut

    gen = torch.Generator().manual_seed(4)
    # 2 x 2 pools of rows with W a multiple of 4 take the 16-byte kernels (odd H too)
    for k, sc, shape in ((2, False, (3, 5, 8, 8)), (4, False, (2, 7, 4, 4)), (2, True, (2, 3, 7, 9)),
                         (2, False, (2, 4, 7, 12)), (2, True, (4, 32, 32, 32))):
        ma, Sa = rnd(gen, *shape), rnd(gen, *shape, kind="u")
        pool = AvgPool2D(k, spatial_correlation=sc)
        om, oS = pool.forward(g(ma), g(Sa))
        rm, rS = F.avgpool_forward(ma, Sa, k, sc)
        assert_rel(om, rm, 1e-6, "pool m")
        assert_rel(oS, rS, 1e-6, "pool S")
        dm, dS = rnd(gen, *om.shape), rnd(gen, *om.shape)
        bm, bS = pool.backward(g(dm), g(dS))
        em, eS = F.avgpool_backward(dm, dS, shape, k, sc)
        assert_rel(bm, em, 1e-7, "pool dm")
        assert_rel(bS, eS, 1e-7, "pool dS")
    a, b = g(rnd(gen, 1001)), g(rnd(gen, 1001))
    a2, b2 = a.clone(), b.clone()
    triton_add_shortcut(a2, b2, a, b)
    assert torch.equal(a, 2 * a2) and torch.equal(b, 2 * b2)


@pytest.mark.parametrize("B,S,E", [(3, 50, 96), (2, 9, 50), (8, 512, 512)])
def test_rmsnorm_against_oracle(B, S, E):
    """Rows of 4-column groups (16-byte path) and not, and the transformer's
    width (column sums by clusters of row slices)."""
    import oracle.net as ON
    from triton_tagi import RMSNorm

    gen = torch.Generator().manual_seed(12)
    ref, dev = ON.RMSNorm(E), RMSNorm(E, device=DEV)
    ref.mw = ref.mw + rnd(gen, E, scale=0.1)
    dev.mw = g(ref.mw)
    ma, Sa = rnd(gen, B, S, E), rnd(gen, B, S, E, kind="u", scale=0.1)
    rm, rS = ref.forward(ma, Sa)
    gm, gS = dev.forward(g(ma), g(Sa))
    assert_rel(gm, rm, 1e-5, "rms mz")
    assert_rel(gS, rS, 1e-4, "rms Sz")
    dm, dS = rnd(gen, B, S, E, scale=0.1), -rnd(gen, B, S, E, kind="u", scale=0.01)
    r = ref.backward(dm, dS)
    d = dev.backward(g(dm), g(dS))
    assert_rel(d[0], r[0], 1e-5, "rms dma")
    assert_rel(d[1], r[1], 1e-4, "rms dSa")
    assert_rel(dev.delta_mw, ref.delta_mw, 1e-5, "rms delta_mw")
    assert_rel(dev.delta_Sw, ref.delta_Sw, 1e-4, "rms delta_Sw")


def test_empty_inputs_are_no_ops():
    from triton_tagi.kernels.common import triton_fused_var_forward
    from triton_tagi.update.parameters import update_parameters

    z = torch.empty(0, 5, device=DEV)
    w = torch.rand(5, 3, device=DEV)
    assert triton_fused_var_forward(z, z, w, w, torch.zeros(1, 3, device=DEV)).shape == (0, 3)
    e = torch.empty(0, device=DEV)
    update_parameters(e, e, e, e, 2.0)


@pytest.mark.parametrize("N,C,H,W", [(8, 16, 6, 6), (3, 5, 7, 5), (16, 64, 8, 8), (16, 512, 4, 4)])
def test_relu_jacobian_folded_into_batchnorm_backward(N, C, H, W):
    """A ReLU feeding a BatchNorm2D, as containers run its backward (the ReLU's
    Jacobian applied by the BatchNorm's backward), against the two layers' own
    backward passes: deltas and parameter deltas."""
    from triton_tagi import BatchNorm2D, ReLU

    gen = torch.Generator().manual_seed(N * C + H)
    mz, Sz = g(rnd(gen, N, C, H, W)), g(rnd(gen, N, C, H, W, kind="u", scale=0.5, lo=1e-3))
    dm, dS = g(rnd(gen, N, C, H, W, scale=0.1)), g(-rnd(gen, N, C, H, W, kind="u", scale=1e-2))
    outs = []
    for fused in (False, True):
        torch.manual_seed(3)
        relu, bn = ReLU(), BatchNorm2D(C, device=DEV)
        ma, Sa = bn.forward(*relu.forward(mz, Sz))
        J = relu.J.clone()
        bn._set_param_mode("deltas")
        if fused:
            dz, dSz = bn.backward(dm, dS, relu=relu)
        else:
            dz, dSz = relu.backward(*bn.backward(dm, dS))
        outs.append((ma, Sa, J, bn.running_mean, bn.running_var, dz, dSz, bn.delta_mw,
                     bn.delta_Sw, bn.delta_mb, bn.delta_Sb))
    names = ("ma", "Sa", "J", "running_mean", "running_var", "d_mz", "d_Sz", "delta_mw",
             "delta_Sw", "delta_mb", "delta_Sb")
    for name, a, b in zip(names, *outs):
        torch.testing.assert_close(b, a, rtol=1e-6, atol=1e-9, msg=name)


@pytest.mark.parametrize("V,D", [(64, 512), (37, 40), (5, 3)])
def test_embedding_against_oracle(V, D):
    """tagi_embedding_forward gathers the rows of every token id; the weight
    deltas of tagi_embedding_backward add the tokens' products in token order,
    the same float32 operations as the oracle's index_add."""
    import oracle.net as ON
    from triton_tagi.layers.embedding import Embedding

    gen = torch.Generator().manual_seed(V * D)
    torch.manual_seed(V)
    ref = ON.Embedding(V, D, scale=0.5)
    dev = Embedding(V, D, scale=0.5, device=DEV)
    dev.mw, dev.Sw = g(ref.mw), g(ref.Sw)
    ids = torch.randint(0, V, (3, 37), generator=gen).float()
    rm, rS = ref.forward(ids, torch.zeros_like(ids))
    mz, Sz = dev.forward(g(ids), g(torch.zeros_like(ids)))
    assert torch.equal(mz.cpu(), rm) and torch.equal(Sz.cpu(), rS)
    dm, dS = rnd(gen, 3, 37, D), -rnd(gen, 3, 37, D, kind="u")
    ref.backward(dm, dS)
    dev.backward(g(dm), g(dS))
    torch.testing.assert_close(dev.delta_mw.cpu(), ref.delta_mw, rtol=1e-6, atol=1e-12)
    torch.testing.assert_close(dev.delta_Sw.cpu(), ref.delta_Sw, rtol=1e-6, atol=1e-12)


def test_embedding_padding_out_of_range_and_sums():
    """Padding and out-of-range ids give zero rows and add nothing; the sums
    mode returns the raw per-row sums (what data parallelism all-reduces)."""
    from triton_tagi._lib import WGRAD_SUMS, lib, stream

    gen = torch.Generator().manual_seed(11)
    V, D, n = 16, 24, 300
    mw, Sw = rnd(gen, V, D), rnd(gen, V, D, kind="u")
    ids = torch.randint(-2, V + 2, (n,), generator=gen).float()
    ids[::7] = 3.0  # padding id
    ids[5] = 2.7    # truncates to 2, as .long()
    dm, dS = rnd(gen, n, D), rnd(gen, n, D)
    d_ids, d_mw, d_Sw, d_dm, d_dS = g(ids), g(mw), g(Sw), g(dm), g(dS)
    mz, Sz = torch.full((n, D), 7.0, device=DEV), torch.full((n, D), 7.0, device=DEV)
    lib()("tagi_embedding_forward", d_ids.data_ptr(), d_mw.data_ptr(), d_Sw.data_ptr(),
          mz.data_ptr(), Sz.data_ptr(), n, V, D, 3, stream(mz))
    cat = ids.long()
    keep = (cat >= 0) & (cat < V) & (cat != 3)
    safe = cat.clamp(0, V - 1)
    ex_m = torch.where(keep[:, None], mw[safe], torch.zeros(()))
    ex_S = torch.where(keep[:, None], Sw[safe], torch.zeros(()))
    assert torch.equal(mz.cpu(), ex_m) and torch.equal(Sz.cpu(), ex_S)
    gm, gS = torch.full((V, D), 7.0, device=DEV), torch.full((V, D), 7.0, device=DEV)
    lib()("tagi_embedding_backward", d_ids.data_ptr(), d_dm.data_ptr(), d_dS.data_ptr(), None,
          n, V, D, 3, WGRAD_SUMS, gm.data_ptr(), gS.data_ptr(), stream(gm))
    w = keep[:, None].float()
    ref_m = torch.zeros(V, D).index_add_(0, safe, dm * w)
    ref_S = torch.zeros(V, D).index_add_(0, safe, dS * w)
    torch.testing.assert_close(gm.cpu(), ref_m, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(gS.cpu(), ref_S, rtol=1e-6, atol=1e-6)


def test_positional_encoding_add():
    """tagi_positional_add adds the table row of each position to the means;
    the variances pass through."""
    from triton_tagi.layers.positional_encoding import PositionalEncoding

    gen = torch.Generator().manual_seed(5)
    pe = PositionalEncoding(48, max_seq_len=64, device=DEV)
    ma, Sa = g(rnd(gen, 3, 20, 48)), g(rnd(gen, 3, 20, 48, kind="u"))
    om, oS = pe.forward(ma, Sa)
    assert torch.equal(om, ma + pe.pe_cache[:20]) and oS is Sa
    with pytest.raises(ValueError):
        pe.forward(g(rnd(gen, 2, 65, 48)), None)


@pytest.mark.parametrize("N,C,H,W,first,residual", [(16, 64, 8, 8, True, False),
                                                      (12, 32, 5, 5, False, True),
                                                      (8, 128, 4, 4, True, True),
                                                      (8, 256, 4, 4, False, True),
                                                      (4, 300, 3, 3, True, False)])
def test_bn_sync_forward_two_shards(N, C, H, W, first, residual):
    """SyncBN on one GPU with two emulated ranks: each half of the batch forms
    its channel sums, the sums are added (the all-reduce), and
    tagi_bn_sync_forward finalises and normalises each half (residual added);
    both halves together equal the oracle's BatchNorm forward on the whole
    batch, and the running statistics follow the reference's init / EMA."""
    from triton_tagi._lib import lib, stream

    L = lib()
    g = torch.Generator().manual_seed(N * C + H)
    mz, Sz = torch.randn(N, C, H, W, generator=g) * 2 + 0.5, torch.rand(N, C, H, W, generator=g)
    rm, rv = torch.randn(C, generator=g), torch.rand(C, generator=g) + 0.5
    mg, Sg = torch.rand(C, generator=g) + 0.5, torch.rand(C, generator=g) * 0.1
    mb, Sb = torch.randn(C, generator=g) * 0.1, torch.rand(C, generator=g) * 0.1
    add_m, add_S = torch.randn(N, C, H, W, generator=g), torch.rand(N, C, H, W, generator=g)
    eps, mom = 1e-5, 0.1
    halves = [slice(0, N // 2), slice(N // 2, N)]
    d = {k: v.to(DEV) for k, v in dict(mz=mz, Sz=Sz, add_m=add_m, add_S=add_S).items()}
    sums = torch.zeros(3 * C, dtype=torch.float64, device=DEV)
    for h in halves:
        part = torch.empty(3 * C, dtype=torch.float64, device=DEV)
        m_h, S_h = d["mz"][h].contiguous(), d["Sz"][h].contiguous()
        L("tagi_bn_channel_sums", m_h.data_ptr(), S_h.data_ptr(), part.data_ptr(), N // 2, C,
          H * W, stream(m_h))
        sums += part
    outs = []
    for h in halves:
        prm = [t.clone().to(DEV) for t in (rm, rv, mg, Sg, mb, Sb)]
        mean, var = torch.empty(C, device=DEV), torch.empty(C, device=DEV)
        m_h, S_h = d["mz"][h].contiguous(), d["Sz"][h].contiguous()
        a_m = d["add_m"][h].contiguous() if residual else None
        a_S = d["add_S"][h].contiguous() if residual else None
        ma, Sa, mh = (torch.empty_like(m_h) for _ in range(3))
        L("tagi_bn_sync_forward", m_h.data_ptr(), S_h.data_ptr(), sums.data_ptr(),
          float(N * H * W), mean.data_ptr(), var.data_ptr(), prm[0].data_ptr(), prm[1].data_ptr(),
          prm[2].data_ptr(), prm[3].data_ptr(), prm[4].data_ptr(), prm[5].data_ptr(),
          ma.data_ptr(), Sa.data_ptr(), mh.data_ptr(),
          a_m.data_ptr() if residual else None, a_S.data_ptr() if residual else None,
          N // 2, C, H * W, 1 if first else 0, 1, mom, eps, stream(m_h))
        outs.append((ma, Sa, mean, var, prm))
    torch.cuda.synchronize()
    e_mean, e_var = F.bn_batch_stats(mz.double(), Sz.double())
    g_ref = torch.sqrt(e_var + eps) if first else mg.double()
    e_ma, e_Sa, _, _ = F.bn_forward(mz.double(), Sz.double(), e_mean, e_var, g_ref, Sg.double(),
                                    mb.double(), Sb.double(), eps)
    if residual:
        e_ma, e_Sa = e_ma + add_m.double(), e_Sa + add_S.double()
    got_m = torch.cat([o[0].cpu() for o in outs])
    got_S = torch.cat([o[1].cpu() for o in outs])
    assert_rel(got_m, e_ma, MEAN_RTOL, "ma")
    assert_rel(got_S, e_Sa, VAR_RTOL, "Sa")
    e_rm = e_mean if first else (1 - mom) * rm.double() + mom * e_mean
    e_rv = e_var if first else (1 - mom) * rv.double() + mom * e_var
    for ma, Sa, mean, var, prm in outs:  # every shard finalises the same statistics
        assert_rel(mean, e_mean, MEAN_RTOL, "mean")
        assert_rel(var, e_var, VAR_RTOL, "var")
        assert_rel(prm[0], e_rm, MEAN_RTOL, "running mean")
        assert_rel(prm[1], e_rv, VAR_RTOL, "running var")
        assert_rel(prm[2], g_ref, MEAN_RTOL, "gamma")
    assert torch.equal(outs[0][2], outs[1][2]) and torch.equal(outs[0][3], outs[1][3])
