"""The tcgen05 (3xTF32) moment contractions against the float64 oracle.

Shapes are chosen so that the library routes them to the tensor-core kernel
(M ≥ 16, N ≥ 16, reduction ≥ 8 and M·N·K ≥ 4e6) and cover ragged tails in
every dimension, operands narrower than one K-block or a quarter tile, the variance-only forward, row-split (NCHW) operand views,
the split reduction of the weight sums, the fused capped update and batched
attention products. Weight sums of at most 96 rows and 64 columns over a
reduction of 16384 or more (the narrow shapes of TC_SHAPES, stem convolutions)
run on the CUDA-core slice kernel instead and are checked the same way. Each
test also checks that no bounded wait inside the kernel ran out
(tagi_device_status).
"""

from __future__ import annotations

import pytest
import torch

import oracle.moments as F
from _tol import MEAN_RTOL, VAR_RTOL, assert_rel

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ok():
    from triton_tagi._lib import device_status

    assert device_status(reset=True) == 0, "a tensor-core kernel wait timed out"


def _rnd(gen, *shape, u=False, scale=1.0, lo=0.0):
    t = torch.rand(*shape, generator=gen) if u else torch.randn(*shape, generator=gen)
    return t * scale + lo


class _on_tensor_cores:
    """The calls inside ran at least ``n`` tcgen05 launches (the library's own
    count of its tensor-core contractions); n = 0: none at all."""

    def __init__(self, n=1):
        self.n = n

    def __enter__(self):
        from triton_tagi._lib import tc_launches

        self.t0 = tc_launches()
        return self

    def __exit__(self, *exc):
        from triton_tagi._lib import tc_launches

        if exc[0] is None:
            ran = tc_launches() - self.t0
            if self.n == 0:
                assert ran == 0, f"{ran} tensor-core launches, expected none"
            else:
                assert ran >= self.n, f"{ran} tensor-core launches, expected at least {self.n}"


TC_SHAPES = [(128, 64, 512), (300, 77, 200), (1000, 576, 64), (2048, 1152, 128),
             (4099, 35, 130), (1555, 256, 17), (131072, 27, 64), (40000, 12, 48), (24, 2048, 512)]


@pytest.mark.parametrize("M,K,N", TC_SHAPES)
def test_forward_full(M, K, N):
    from triton_tagi import Linear
    from triton_tagi.kernels.common import triton_fused_var_forward

    g = torch.Generator().manual_seed(M + K + N)
    ma, Sa = _rnd(g, M, K), _rnd(g, M, K, u=True, scale=1e-2, lo=1e-4)
    mw, Sw = _rnd(g, K, N, scale=K**-0.5), _rnd(g, K, N, u=True, scale=1.0 / K)
    mb, Sb = _rnd(g, 1, N, scale=0.1), _rnd(g, 1, N, u=True, scale=1e-3)
    lin = Linear(K, N, device=DEV)
    lin.mw, lin.Sw, lin.mb, lin.Sb = (t.to(DEV) for t in (mw, Sw, mb, Sb))
    with _on_tensor_cores():
        mz, Sz = lin.forward(ma.to(DEV), Sa.to(DEV))
    d = lambda t: t.double()  # noqa: E731
    assert_rel(mz, F.mean_forward(d(ma), d(mw), d(mb)), MEAN_RTOL, "mz")
    ref_S = F.var_forward(d(ma), d(Sa), d(mw), d(Sw), d(Sb))
    assert_rel(Sz, ref_S, VAR_RTOL, "Sz")
    only = triton_fused_var_forward(ma.to(DEV), Sa.to(DEV), mw.to(DEV), Sw.to(DEV), Sb.to(DEV))
    assert_rel(only, ref_S, VAR_RTOL, "Sz (variance only)")
    _ok()


@pytest.mark.parametrize("M,K,N", TC_SHAPES)
def test_backward_delta_and_weight_sums(M, K, N):
    from triton_tagi.kernels.common import triton_fused_backward_delta, triton_fused_weight_grad

    g = torch.Generator().manual_seed(3 * M + N)
    a, mw = _rnd(g, M, K), _rnd(g, K, N, scale=K**-0.5)
    dmz, dSz = _rnd(g, M, N, scale=0.1), -_rnd(g, M, N, u=True, scale=1e-2)
    # input deltas K wide: outputs narrower than 16 columns run on CUDA cores
    with _on_tensor_cores(1 if K >= 16 else 0):
        d_ma, d_Sa = triton_fused_backward_delta(dmz.to(DEV), dSz.to(DEV), mw.to(DEV))
    r_ma, r_Sa = F.backward_delta(dmz.double(), dSz.double(), mw.double())
    assert_rel(d_ma, r_ma, MEAN_RTOL, "d_ma")
    assert_rel(d_Sa, r_Sa, VAR_RTOL, "d_Sa")
    # weight sums of a few rows and columns over a long reduction (network
    # stems: 27 x 64 over 131072 pixels) run on the CUDA-core kernel by design
    stem = K <= 96 and N <= 64 and M >= 16384
    with _on_tensor_cores(0 if stem else 1):
        gm, gS = triton_fused_weight_grad(a.to(DEV), dmz.to(DEV), dSz.to(DEV))
    rm, rS = F.weight_grad(a.double(), dmz.double(), dSz.double())
    assert_rel(gm, rm, MEAN_RTOL, "grad_mw")
    assert_rel(gS, rS, VAR_RTOL, "grad_Sw")
    _ok()


def test_weight_sums_long_reduction_split():
    from triton_tagi.kernels.common import triton_fused_weight_grad

    g = torch.Generator().manual_seed(11)
    a, dmz, dSz = _rnd(g, 60000, 300), _rnd(g, 60000, 64), _rnd(g, 60000, 64, u=True)
    gm, gS = triton_fused_weight_grad(a.to(DEV), dmz.to(DEV), dSz.to(DEV))
    rm, rS = F.weight_grad(a.double(), dmz.double(), dSz.double())
    assert_rel(gm, rm, MEAN_RTOL, "grad_mw")
    assert_rel(gS, rS, VAR_RTOL, "grad_Sw")
    _ok()


@pytest.mark.parametrize("M,K,N", [(256, 4096, 1024), (96, 3000, 600), (32, 2048, 512)])
def test_linear_entries_split_reduction(M, K, N):
    """tagi_linear_forward / tagi_linear_backward_delta with the workspace the
    library asks for (the reduction split over idle SMs, partials added in split
    order) and without one (unsplit): both against the float64 oracle. The last
    shape runs on the CUDA-core kernel."""
    from triton_tagi._lib import lib, stream, workspace

    L = lib()
    g = torch.Generator().manual_seed(M + 7 * K + N)
    ma, Sa = _rnd(g, M, K), _rnd(g, M, K, u=True, scale=1e-2, lo=1e-4)
    mw, Sw = _rnd(g, K, N, scale=K**-0.5), _rnd(g, K, N, u=True, scale=1.0 / K)
    mb, Sb = _rnd(g, N, scale=0.1), _rnd(g, N, u=True, scale=1e-3)
    dmz, dSz = _rnd(g, M, N, scale=0.1), -_rnd(g, M, N, u=True, scale=1e-2)
    dv = [t.to(DEV) for t in (ma, Sa, mw, Sw, mb, Sb, dmz, dSz)]
    d = lambda t: t.double()  # noqa: E731
    ex_m = F.mean_forward(d(ma), d(mw), d(mb).view(1, -1))
    ex_S = F.var_forward(d(ma), d(Sa), d(mw), d(Sw), d(Sb).view(1, -1))
    r_ma, r_Sa = F.backward_delta(d(dmz), d(dSz), d(mw))
    nf = L.size("tagi_store_workspace_size", M, N, K)
    nb = L.size("tagi_store_workspace_size", M, K, N)
    assert nf > 0 and nb > 0, "shape chosen to split the reduction"
    for split in (True, False):
        mz, Sz = torch.empty(M, N, device=DEV), torch.empty(M, N, device=DEV)
        hold, wp, wn = workspace(nf if split else 0, mz)
        L("tagi_linear_forward", *(t.data_ptr() for t in dv[:6]), mz.data_ptr(), Sz.data_ptr(),
          M, K, N, wp, wn, stream(mz))
        d_ma, d_Sa = torch.empty(M, K, device=DEV), torch.empty(M, K, device=DEV)
        hold2, wp, wn = workspace(nb if split else 0, mz)
        L("tagi_linear_backward_delta", dv[6].data_ptr(), dv[7].data_ptr(), dv[2].data_ptr(),
          d_ma.data_ptr(), d_Sa.data_ptr(), M, K, N, wp, wn, stream(mz))
        assert_rel(mz, ex_m, MEAN_RTOL, f"mz split={split}")
        assert_rel(Sz, ex_S, VAR_RTOL, f"Sz split={split}")
        assert_rel(d_ma, r_ma, MEAN_RTOL, f"d_ma split={split}")
        assert_rel(d_Sa, r_Sa, VAR_RTOL, f"d_Sa split={split}")
        _ok()


def test_conv_layer_small_maps_split_reduction():
    """A late-stage Conv2D (4x4 maps, 256 channels): the forward and stride-1
    input-delta contractions leave SMs idle, so the layer passes the library's
    workspace and the reduction over (tap, channel) is split."""
    import oracle.net as ON
    from triton_tagi import Conv2D
    from triton_tagi._lib import lib

    C = Co = 256
    N, H, W, k = 8, 4, 4, 3
    assert lib().size("tagi_store_workspace_size", N * H * W, Co, C * k * k) > 0
    assert lib().size("tagi_store_workspace_size", N * H * W, C, Co * k * k) > 0
    g = torch.Generator().manual_seed(12)
    torch.manual_seed(6)
    ref = ON.Conv2D(C, Co, k, 1, 1, 1)
    dev = Conv2D(C, Co, k, 1, 1, 1, device=DEV)
    for n in ("mw", "Sw", "mb", "Sb"):
        setattr(dev, n, getattr(ref, n).to(DEV))
    ma, Sa = _rnd(g, N, C, H, W), _rnd(g, N, C, H, W, u=True, scale=0.1)
    d = lambda t: t.double()  # noqa: E731
    ex_m, ex_S, _ = F.conv_forward(d(ma), d(Sa), d(ref.mw), d(ref.Sw), d(ref.mb), d(ref.Sb),
                                   k, 1, 1, 1)
    mz, Sz = dev.forward(ma.to(DEV), Sa.to(DEV))
    assert_rel(mz, ex_m, MEAN_RTOL, "mz")
    assert_rel(Sz, ex_S, VAR_RTOL, "Sz")
    ref.forward(ma, Sa)
    dmz, dSz = _rnd(g, *ex_m.shape, scale=0.1), -_rnd(g, *ex_m.shape, u=True, scale=1e-2)
    r_dm, r_dS = ref.backward(dmz, dSz)
    d_dm, d_dS = dev.backward(dmz.to(DEV), dSz.to(DEV))
    assert_rel(d_dm, r_dm, MEAN_RTOL, "d_ma")
    assert_rel(d_dS, r_dS, VAR_RTOL, "d_Sa")
    _ok()


@pytest.mark.parametrize("mode", ["deltas", "update"])
def test_linear_parameter_epilogue(mode):
    import oracle.net as ON
    from triton_tagi import Linear

    g = torch.Generator().manual_seed(5)
    M, K, N = 512, 600, 96
    torch.manual_seed(1)
    ref = ON.Linear(K, N)
    dev = Linear(K, N, device=DEV)
    for n in ("mw", "Sw", "mb", "Sb"):
        setattr(dev, n, getattr(ref, n).to(DEV))
    ma = _rnd(g, M, K)
    ref.forward(ma, torch.zeros_like(ma))
    dev.forward(ma.to(DEV), torch.zeros(M, K, device=DEV))
    dm, dS = _rnd(g, M, N, scale=0.1), -_rnd(g, M, N, u=True, scale=1e-2)
    ref.backward(dm, dS)
    prev_S = ref.Sw.clone()
    dev._set_param_mode(mode, 3.0)
    dev.backward(dm.to(DEV), dS.to(DEV))
    if mode == "deltas":
        assert_rel(dev.delta_mw, ref.delta_mw, MEAN_RTOL, "delta_mw")
        assert_rel(dev.delta_Sw, ref.delta_Sw, VAR_RTOL, "delta_Sw")
        assert_rel(dev.delta_mb, ref.delta_mb, MEAN_RTOL, "delta_mb")
    else:
        ref.update(3.0)
        assert_rel(dev.mw, ref.mw, MEAN_RTOL, "mw")
        from _tol import var_update_err

        assert var_update_err(dev.Sw, ref.Sw, prev_S) <= VAR_RTOL
    dev._set_param_mode("deltas")
    _ok()


def test_conv_layer_nchw_views_on_tensor_cores():
    import oracle.net as ON
    from triton_tagi import Conv2D

    g = torch.Generator().manual_seed(8)
    N, C, H, W, Co = 8, 16, 16, 16, 32  # M = 2048, K = 144, N = 32
    torch.manual_seed(2)
    ref = ON.Conv2D(C, Co, 3, 1, 1, 1)
    dev = Conv2D(C, Co, 3, 1, 1, 1, device=DEV)
    for n in ("mw", "Sw", "mb", "Sb"):
        setattr(dev, n, getattr(ref, n).to(DEV))
    ma, Sa = _rnd(g, N, C, H, W), _rnd(g, N, C, H, W, u=True, scale=0.1)
    rm, rS = ref.forward(ma, Sa)
    dm_, dS_ = dev.forward(ma.to(DEV), Sa.to(DEV))
    assert_rel(dm_, rm, MEAN_RTOL, "conv mz")
    assert_rel(dS_, rS, VAR_RTOL, "conv Sz")
    dmz, dSz = _rnd(g, *rm.shape, scale=0.1), -_rnd(g, *rm.shape, u=True, scale=1e-2)
    r = ref.backward(dmz, dSz)
    d = dev.backward(dmz.to(DEV), dSz.to(DEV))
    assert_rel(d[0], r[0], MEAN_RTOL, "conv d_ma")
    assert_rel(d[1], r[1], VAR_RTOL, "conv d_Sa")
    assert_rel(dev.delta_mw, ref.delta_mw, MEAN_RTOL, "conv delta_mw")
    assert_rel(dev.delta_Sw, ref.delta_Sw, VAR_RTOL, "conv delta_Sw")
    _ok()


def test_batched_attention_products():
    from triton_tagi.kernels.attention import bmm_shared_left, bmm_shared_right, bmm_tagi_moments

    g = torch.Generator().manual_seed(21)
    B, H, S, D = 2, 4, 256, 64
    mq, Sq = _rnd(g, B, H, S, D), _rnd(g, B, H, S, D, u=True, scale=0.1)
    mk, Sk = _rnd(g, B, H, S, D), _rnd(g, B, H, S, D, u=True, scale=0.1)
    s = D**-0.5
    tr = lambda t: t.transpose(-1, -2)  # noqa: E731
    m, v = bmm_tagi_moments(mq.to(DEV), Sq.to(DEV), tr(mk.to(DEV)), tr(Sk.to(DEV)), s, s * s)
    assert_rel(m, s * (mq.double() @ tr(mk.double())), MEAN_RTOL, "scores mean")
    assert_rel(v, F.bmm_tagi_var(mq.double(), Sq.double(), tr(mk.double()), tr(Sk.double()), s * s),
               VAR_RTOL, "scores var")
    dm, dv = _rnd(g, B, H, S, S, scale=0.1), _rnd(g, B, H, S, S, u=True, scale=0.01)
    m, v = bmm_shared_right(dm.to(DEV), dv.to(DEV), mk.to(DEV), scale=s)
    rm, rv = F.bmm_shared_right(dm.double(), dv.double(), mk.double(), s)
    assert_rel(m, rm, MEAN_RTOL, "shared right mean")
    assert_rel(v, rv, VAR_RTOL, "shared right var")
    m, v = bmm_shared_left(tr(dm.to(DEV)), mk.to(DEV), Sk.to(DEV))
    rm, rv = F.bmm_shared_left(tr(dm.double()), mk.double(), Sk.double())
    assert_rel(m, rm, MEAN_RTOL, "shared left mean")
    assert_rel(v, rv, VAR_RTOL, "shared left var")
    # left operand with contiguous rows: the 64-column tensor-memory tiles
    m, v = bmm_shared_left(dm.to(DEV), mk.to(DEV), Sk.to(DEV), 0.5)
    rm, rv = F.bmm_shared_left(dm.double(), mk.double(), Sk.double(), 0.5)
    assert_rel(m, rm, MEAN_RTOL, "shared left mean (row-contiguous a)")
    assert_rel(v, rv, VAR_RTOL, "shared left var (row-contiguous a)")
    _ok()


@pytest.mark.parametrize("C,Co,k,p", [(64, 64, 3, 1), (128, 96, 3, 1), (40, 72, 5, 2),
                                      (64, 64, 3, 0), (96, 64, 1, 0)])
def test_conv_stride1_input_deltas_as_one_contraction(C, Co, k, p):
    """Conv2D.backward gathers the deltas as the col2im fold does inside one
    contraction (tagi_conv2d_backward_delta); at stride 1 it must equal the
    reference's patch-space product followed by its col2im gather."""
    import oracle.net as ON
    from triton_tagi import Conv2D

    g = torch.Generator().manual_seed(C + Co + k)
    N, H, W = 4, 14, 13
    torch.manual_seed(3)
    ref = ON.Conv2D(C, Co, k, 1, p, 1)
    dev = Conv2D(C, Co, k, 1, p, 1, device=DEV)
    for n in ("mw", "Sw", "mb", "Sb"):
        setattr(dev, n, getattr(ref, n).to(DEV))
    ma, Sa = _rnd(g, N, C, H, W), _rnd(g, N, C, H, W, u=True, scale=0.1)
    rm, _ = ref.forward(ma, Sa)
    dev.forward(ma.to(DEV), Sa.to(DEV))
    dmz, dSz = _rnd(g, *rm.shape, scale=0.1), -_rnd(g, *rm.shape, u=True, scale=1e-2)
    r_dm, r_dS = ref.backward(dmz, dSz)
    d_dm, d_dS = dev.backward(dmz.to(DEV), dSz.to(DEV))
    patches = F.im2col(ma.double(), k, 1, p, 1)
    exact_m, exact_S = F.conv_backward(dmz.double(), dSz.double(), patches, ref.mw.double(),
                                       (N, C, H, W), k, 1, p, 1)[:2]
    assert_rel(d_dm, exact_m, MEAN_RTOL, "d_ma vs float64")
    assert_rel(d_dS, exact_S, VAR_RTOL, "d_Sa vs float64")
    assert_rel(d_dm, r_dm, MEAN_RTOL, "d_ma vs reference restatement")
    assert_rel(d_dS, r_dS, VAR_RTOL, "d_Sa vs reference restatement")
    # weight deltas from the channels-last copy of the deltas (Co % 8 == 0)
    assert_rel(dev.delta_mw, ref.delta_mw, MEAN_RTOL, "delta_mw")
    assert_rel(dev.delta_Sw, ref.delta_Sw, VAR_RTOL, "delta_Sw")
    assert_rel(dev.delta_mb, ref.delta_mb, MEAN_RTOL, "delta_mb")
    assert_rel(dev.delta_Sb, ref.delta_Sb, VAR_RTOL, "delta_Sb")
    _ok()


@pytest.mark.parametrize("C,Co,k,s,p,pt", [(64, 128, 3, 2, 1, 1), (32, 64, 5, 1, 2, 2),
                                           (48, 80, 3, 1, 1, 1), (64, 64, 1, 2, 0, 1)])
def test_conv_layer_gathered_patches(C, Co, k, s, p, pt):
    """Conv2D.forward gathers its patches inside the contraction
    (tagi_conv2d_forward); forward, input deltas and weight deltas against the
    float64 oracle, at sizes that run on the tensor cores."""
    import oracle.net as ON
    from triton_tagi import Conv2D

    g = torch.Generator().manual_seed(C * k + Co + s)
    N, H, W = 6, 15, 12
    torch.manual_seed(4)
    ref = ON.Conv2D(C, Co, k, s, p, pt)
    dev = Conv2D(C, Co, k, s, p, pt, device=DEV)
    for n in ("mw", "Sw", "mb", "Sb"):
        setattr(dev, n, getattr(ref, n).to(DEV))
    ma, Sa = _rnd(g, N, C, H, W), _rnd(g, N, C, H, W, u=True, scale=0.1)
    d = lambda t: t.double()  # noqa: E731
    ex_m, ex_S, patches = F.conv_forward(d(ma), d(Sa), d(ref.mw), d(ref.Sw), d(ref.mb), d(ref.Sb),
                                         k, s, p, pt)
    ref.forward(ma, Sa)
    mz, Sz = dev.forward(ma.to(DEV), Sa.to(DEV))
    assert_rel(mz, ex_m, MEAN_RTOL, "mz")
    assert_rel(Sz, ex_S, VAR_RTOL, "Sz")
    dmz, dSz = _rnd(g, *ex_m.shape, scale=0.1), -_rnd(g, *ex_m.shape, u=True, scale=1e-2)
    for mode in ("reference", "adjoint"):  # the two col2im gathers differ for stride > 1
        dev.col2im_mode = mode
        ref.col2im_adjoint = mode == "adjoint"
        ref.forward(ma, Sa)
        dev.forward(ma.to(DEV), Sa.to(DEV))
        r_dm, r_dS = ref.backward(dmz, dSz)
        d_dm, d_dS = dev.backward(dmz.to(DEV), dSz.to(DEV))
        assert_rel(d_dm, r_dm, MEAN_RTOL, f"d_ma {mode}")
        assert_rel(d_dS, r_dS, VAR_RTOL, f"d_Sa {mode}")
        assert_rel(dev.delta_mw, ref.delta_mw, MEAN_RTOL, "delta_mw")
        assert_rel(dev.delta_Sw, ref.delta_Sw, VAR_RTOL, "delta_Sw")
    _ok()


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("C,Co,k,s,p,pt", [(32, 64, 3, 2, 1, 1), (16, 48, 2, 2, 0, 1),
                                           (24, 32, 3, 2, 1, 2)])
def test_conv_backward_delta_entry_strided_gathers(C, Co, k, s, p, pt, mode):
    """tagi_conv2d_backward_delta with stride > 1: the reference's col2im gather
    (mode 0, no column-divisibility test) and the adjoint (mode 1), against the
    oracle's patch-space product followed by the same gather."""
    from triton_tagi._lib import lib, stream

    g = torch.Generator().manual_seed(C + Co + k + s + mode)
    N, H, W = 4, 17, 14
    mw = _rnd(g, C * k * k, Co, scale=(C * k * k) ** -0.5)
    Ho, Wo = F.conv_out_hw(H, W, k, s, p, pt)
    dmz, dSz = _rnd(g, N, Co, Ho, Wo, scale=0.1), -_rnd(g, N, Co, Ho, Wo, u=True, scale=1e-2)
    d_dmz, d_dSz, d_mw = dmz.to(DEV), dSz.to(DEV), mw.to(DEV)
    d_ma = torch.empty(N, C, H, W, device=DEV)
    d_Sa = torch.empty_like(d_ma)
    lib()("tagi_conv2d_backward_delta", d_dmz.data_ptr(), d_dSz.data_ptr(), d_mw.data_ptr(),
          d_ma.data_ptr(), d_Sa.data_ptr(), N, C, H, W, Co, k, s, p, pt, mode, 0, None, 0,
          stream(d_ma))
    dm = dmz.double().permute(0, 2, 3, 1).reshape(-1, Co)
    dS = dSz.double().permute(0, 2, 3, 1).reshape(-1, Co)
    dpm, dpS = F.backward_delta(dm, dS, mw.double())
    ref_m = F.col2im(dpm, N, C, H, W, k, s, p, pt, adjoint=mode == 1)
    ref_S = F.col2im(dpS, N, C, H, W, k, s, p, pt, adjoint=mode == 1)
    assert_rel(d_ma, ref_m, MEAN_RTOL, "d_ma")
    assert_rel(d_Sa, ref_S, VAR_RTOL, "d_Sa")
    _ok()


@pytest.mark.parametrize("C,Co", [(16, 24), (12, 20), (64, 64)])
def test_conv_entries_channels_last_equal_nchw(C, Co):
    """tagi_conv2d_forward / tagi_conv2d_backward_delta given the gathered
    tensor channels-last (tagi_nchw_to_nhwc) read the same values in the same
    order as from NCHW: bit-identical outputs, with C a multiple of 8 (one
    32-byte load per tap and operand) and not (element by element)."""
    from triton_tagi._lib import lib, stream

    L = lib()
    g = torch.Generator().manual_seed(C + Co)
    N, H, W, k = 4, 12, 10, 3
    x = [t.to(DEV) for t in (_rnd(g, N, C, H, W), _rnd(g, N, C, H, W, u=True, scale=0.1))]
    mw = _rnd(g, C * k * k, Co, scale=(C * k * k) ** -0.5).to(DEV)
    Sw = _rnd(g, C * k * k, Co, u=True, scale=1e-2).to(DEV)
    mb, Sb = _rnd(g, Co, scale=0.1).to(DEV), _rnd(g, Co, u=True, scale=1e-3).to(DEV)
    d = [t.to(DEV) for t in (_rnd(g, N, Co, H, W, scale=0.1), -_rnd(g, N, Co, H, W, u=True, scale=1e-2))]

    def nhwc(a, b, c):
        ya, yb = torch.empty(N, H, W, c, device=DEV), torch.empty(N, H, W, c, device=DEV)
        L("tagi_nchw_to_nhwc", a.data_ptr(), b.data_ptr(), ya.data_ptr(), yb.data_ptr(), N, c,
          H * W, stream(a))
        assert torch.equal(ya, a.permute(0, 2, 3, 1)) and torch.equal(yb, b.permute(0, 2, 3, 1))
        return ya, yb

    outs = []
    for last in (0, 1):
        xm, xS = nhwc(*x, C) if last else x
        mz, Sz = torch.empty(N, Co, H, W, device=DEV), torch.empty(N, Co, H, W, device=DEV)
        L("tagi_conv2d_forward", xm.data_ptr(), xS.data_ptr(), mw.data_ptr(), Sw.data_ptr(),
          mb.data_ptr(), Sb.data_ptr(), mz.data_ptr(), Sz.data_ptr(), N, C, H, W, Co, k, 1, 1, 1,
          last, None, 0, stream(mz))
        dm, dS = nhwc(*d, Co) if last else d
        da, dA = torch.empty(N, C, H, W, device=DEV), torch.empty(N, C, H, W, device=DEV)
        L("tagi_conv2d_backward_delta", dm.data_ptr(), dS.data_ptr(), mw.data_ptr(), da.data_ptr(),
          dA.data_ptr(), N, C, H, W, Co, k, 1, 1, 1, 0, last, None, 0, stream(da))
        outs.append((mz, Sz, da, dA))
    for name, a, b in zip(("mz", "Sz", "d_ma", "d_Sa"), *outs):
        assert torch.equal(a, b), name
    _ok()


@pytest.mark.parametrize("C,H,W,k,s,p,pt,Co", [(64, 32, 32, 3, 1, 1, 1, 64), (3, 32, 32, 3, 1, 1, 1, 64),
                                              (16, 17, 13, 3, 2, 1, 2, 32), (8, 20, 24, 5, 1, 2, 1, 40)])
def test_param_grad_transposed_patches(C, H, W, k, s, p, pt, Co):
    """tagi_im2col_t writes the transpose of tagi_im2col's patches (bit-exact
    against the oracle's unfold), and tagi_param_grad_t on them gives the
    weight and bias deltas of tagi_param_grad on the plain patches: the
    same reduction in the same order, bit-identical."""
    from triton_tagi._lib import WGRAD_DELTAS, lib, stream

    L = lib()
    g = torch.Generator().manual_seed(C * H + Co)
    N = 8 if C > 8 else 4
    Ho, Wo = F.conv_out_hw(H, W, k, s, p, pt)
    M, K = N * Ho * Wo, C * k * k
    assert M % 8 == 0
    x = _rnd(g, N, C, H, W)
    xd = x.to(DEV)
    pm = torch.empty(M, K, device=DEV)
    L("tagi_im2col", xd.data_ptr(), None, pm.data_ptr(), None, N, C, H, W, k, s, p, pt, stream(xd))
    ptr = torch.full((K, M), 7.0, device=DEV)
    L("tagi_im2col_t", xd.data_ptr(), ptr.data_ptr(), N, C, H, W, k, s, p, pt, stream(xd))
    ref = F.im2col(x, k, s, p, pt)
    assert torch.equal(ptr.cpu(), ref.t().contiguous())
    assert torch.equal(pm.cpu(), ref)
    dmz = _rnd(g, N, Co, Ho, Wo, scale=0.1).to(DEV)
    dSz = -_rnd(g, N, Co, Ho, Wo, u=True, scale=1e-2).to(DEV)
    Sw = _rnd(g, K, Co, u=True, scale=1e-2).to(DEV)
    Sb = _rnd(g, 1, Co, u=True, scale=1e-3).to(DEV)
    d_map = (Ho * Wo, Co * Ho * Wo, 1, Ho * Wo)
    ws = torch.empty(max(L.size("tagi_param_grad_workspace_size", M, K, Co, 1), 1),
                     dtype=torch.uint8, device=DEV)
    outs = []
    for entry, a, lda in (("tagi_param_grad", pm, K), ("tagi_param_grad_t", ptr, M)):
        o = [torch.empty(K, Co, device=DEV), torch.empty(K, Co, device=DEV),
             torch.empty(1, Co, device=DEV), torch.empty(1, Co, device=DEV)]
        L(entry, a.data_ptr(), lda, dmz.data_ptr(), dSz.data_ptr(), *d_map, M, K, Co, 1,
          WGRAD_DELTAS, None, Sw.data_ptr(), None, Sb.data_ptr(), *(t.data_ptr() for t in o), 1.0,
          ws.data_ptr(), ws.numel(), stream(a))
        outs.append(o)
    for name, a, b in zip(("delta_mw", "delta_Sw", "delta_mb", "delta_Sb"), *outs):
        assert torch.equal(a, b), name
    # and against the float64 oracle
    d = lambda t: t.double().cpu()  # noqa: E731
    P = d(ref)
    Dm = d(dmz).permute(0, 2, 3, 1).reshape(M, Co)
    DS = d(dSz).permute(0, 2, 3, 1).reshape(M, Co)
    assert_rel(outs[1][0], d(Sw) * (P.t() @ Dm), MEAN_RTOL, "delta_mw")
    assert_rel(outs[1][1], d(Sw) ** 2 * ((P * P).t() @ DS), VAR_RTOL, "delta_Sw")
    _ok()


@pytest.mark.parametrize("C,Co,k,p,N", [(3, 64, 3, 1, 20), (3, 32, 5, 2, 16), (4, 24, 3, 1, 17)])
def test_stem_weight_sums(C, Co, k, p, N):
    """Weight deltas of stem convolutions: few weight rows (C*k*k + 1 <= 96)
    over a reduction of >= 16384 output pixels, which run on the CUDA-core
    kernel that keeps all outputs of a reduction slice in registers, against
    the float64 oracle (bias included; a pixel count that is not a multiple of
    the staged tile)."""
    import oracle.net as ON
    from triton_tagi import Conv2D

    g = torch.Generator().manual_seed(C * Co + k)
    H = W = 32
    torch.manual_seed(5)
    ref = ON.Conv2D(C, Co, k, 1, p, 1)
    dev = Conv2D(C, Co, k, 1, p, 1, device=DEV)
    for n in ("mw", "Sw", "mb", "Sb"):
        setattr(dev, n, getattr(ref, n).to(DEV))
    ma, Sa = _rnd(g, N, C, H, W), _rnd(g, N, C, H, W, u=True, scale=0.1)
    rm, _ = ref.forward(ma, Sa)
    dev.forward(ma.to(DEV), Sa.to(DEV))
    dmz, dSz = _rnd(g, *rm.shape, scale=0.1), -_rnd(g, *rm.shape, u=True, scale=1e-2)
    ref.backward(dmz, dSz)
    dev._skip_input_delta = True
    dev.backward(dmz.to(DEV), dSz.to(DEV))
    assert_rel(dev.delta_mw, ref.delta_mw, MEAN_RTOL, "delta_mw")
    assert_rel(dev.delta_Sw, ref.delta_Sw, VAR_RTOL, "delta_Sw")
    assert_rel(dev.delta_mb, ref.delta_mb, MEAN_RTOL, "delta_mb")
    assert_rel(dev.delta_Sb, ref.delta_Sb, VAR_RTOL, "delta_Sb")
    _ok()


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("M,K,N", [(3000, 512, 200), (20000, 256, 96), (4096, 512, 512)])
def test_bias_sums_apart_equal_ones_row(M, K, N, mode):
    """With K a multiple of 256 and a workspace of the size the query reports,
    the bias sums are formed by a column-sum pass next to the K-row contraction;
    with a smaller workspace that still holds the plan of K + 1 rows (sized by
    the no-bias query for K + 1) the bias stays a row of ones in the contraction.
    The two agree (sums, deltas and the capped update) and match float64."""
    from triton_tagi._lib import lib, stream

    L = lib()
    g = torch.Generator().manual_seed(M + K + N + mode)
    a = _rnd(g, M, K).to(DEV)
    dmz = _rnd(g, M, N, scale=0.1).to(DEV)
    dSz = -_rnd(g, M, N, u=True, scale=1e-2).to(DEV)
    mw, Sw = _rnd(g, K, N, scale=0.1), _rnd(g, K, N, u=True, scale=1e-2, lo=1e-3)
    mb, Sb = _rnd(g, 1, N, scale=0.1), _rnd(g, 1, N, u=True, scale=1e-2, lo=1e-3)
    need = L.size("tagi_param_grad_workspace_size", M, K, N, 1)
    ones = L.size("tagi_fused_weight_grad_workspace_size", M, K + 1, N)
    assert 0 < ones < need
    outs = []
    for ws_bytes in (need, ones):
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        p = [t.to(DEV).clone() for t in (mw, Sw, mb, Sb)]
        o = [torch.zeros(K + 1, N, device=DEV), torch.zeros(K + 1, N, device=DEV),
             torch.zeros(1, N, device=DEV), torch.zeros(1, N, device=DEV)]
        if mode == 0:
            args = (None, None, None, None, o[0].data_ptr(), o[1].data_ptr(), None, None)
        elif mode == 1:
            args = (None, p[1].data_ptr(), None, p[3].data_ptr(), o[0].data_ptr(),
                    o[1].data_ptr(), o[2].data_ptr(), o[3].data_ptr())
        else:
            args = tuple(t.data_ptr() for t in p) + (None, None, None, None)
        L("tagi_param_grad", a.data_ptr(), K, dmz.data_ptr(), dSz.data_ptr(), 0, 0, N, 1, M, K,
          N, 1, mode, *args, 2.0, ws.data_ptr(), ws_bytes, stream(a))
        outs.append((o, p))
    (o1, p1), (o2, p2) = outs
    if mode == 0:
        gm = (a.double().t() @ dmz.double())
        gS = ((a.double() ** 2).t() @ dSz.double())
        for o in (o1, o2):
            assert_rel(o[0][:K], gm, MEAN_RTOL, "weight sums")
            assert_rel(o[1][:K], gS, VAR_RTOL, "weight var sums")
            assert_rel(o[0][K], dmz.double().sum(0), MEAN_RTOL, "bias sums")
            assert_rel(o[1][K], dSz.double().sum(0), VAR_RTOL, "bias var sums")
    elif mode == 1:
        for x, y in zip(o1, o2):
            assert_rel(x, y.double(), MEAN_RTOL, "deltas")
        assert_rel(o1[2], Sb.double().to(DEV) * dmz.double().sum(0), MEAN_RTOL, "bias delta")
    else:
        for x, y in zip(p1, p2):
            assert_rel(x, y.double(), VAR_RTOL, "updated parameters")
    _ok()
