"""Layer-level parity of the composite layers: ResBlock and MultiheadAttentionV2.

Each layer runs forward, backward and update on its own (the reference's call
structure: deltas stored by backward, applied by update) and is compared with
the oracle's layer in float32 and float64 at the north-star bar: means
normwise ≤ 1e-5, variances and variance deltas element-wise ≤ 1e-4 (with the
reference's own float32 error as the allowance where that is larger, as for
the ReLU variance inside the block), updated variances element-wise ≤ 1e-4 of
the pre-update variance. The cases follow the reference's validation tests
(tests/validation/test_resblock.py:75-302: identity and projection blocks,
forward, input deltas, updates; tests/validation/test_attention.py:328-398,
445-464, 523-560: attention forward, zero deltas, score rows).
"""

from __future__ import annotations

import pytest
import torch

import oracle.moments as F
import oracle.net as ON
import triton_tagi as TT
from _nets import load, params
from _tol import MEAN_RTOL, VAR_RTOL, elem_check, norm_check, var_update_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _check(what, got, r32, r64):
    w, fb, e = norm_check(got[0], r32[0], r64[0], MEAN_RTOL)
    assert w <= 1.0, f"{what} mean: normwise {e:.3e}"
    w, nfb, e = elem_check(got[1], r32[1], r64[1], VAR_RTOL)
    assert w <= 1.0, f"{what} var: element-wise {e:.3e} ({nfb} on the float64 allowance)"
    return e


def _triple(make_ref, make_dev):
    torch.manual_seed(0)
    r32, r64 = make_ref(), make_ref()
    dev = make_dev()
    arrays = [t.numpy() for t in params([r32])]
    load([dev], arrays, device=DEV)
    load([r64], arrays, dtype=torch.float64)
    return dev, r32, r64


def _layer_step(dev, r32, r64, ma, Sa, dm, dS, cap):
    h32 = lambda t: t.float()  # noqa: E731
    h64 = lambda t: t.double()  # noqa: E731
    out = dev.forward(ma.to(DEV), Sa.to(DEV))
    _check("forward", out, r32.forward(h32(ma), h32(Sa)), r64.forward(h64(ma), h64(Sa)))
    back = dev.backward(dm.to(DEV), dS.to(DEV))
    _check("backward", back, r32.backward(h32(dm), h32(dS)), r64.backward(h64(dm), h64(dS)))
    prev = [t.detach().cpu().double() for t in params([dev])]
    dev.update(cap)
    r32.update(cap)
    r64.update(cap)
    got, e32, e64 = params([dev]), params([r32]), params([r64])
    names = [n for leaf in TT_leaves(dev) for n in _pnames(leaf)]
    for n, g, a, b, p in zip(names, got, e32, e64, prev):
        if n in ("Sw", "Sb"):
            e = var_update_err(g, a, p)
            assert e <= VAR_RTOL, f"updated {n}: {e:.3e} of the pre-update variance"
        elif n == "running_var":
            w, _, e = elem_check(g, a, b, VAR_RTOL)
            assert w <= 1.0, f"running_var: {e:.3e}"
        else:
            w, _, e = norm_check(g, a, b, MEAN_RTOL)
            assert w <= 1.0, f"updated {n}: {e:.3e}"
    torch.cuda.synchronize()


def TT_leaves(layer):
    if hasattr(layer, "_learnable"):
        return list(layer._learnable)
    if hasattr(layer, "q_proj"):
        return [layer.q_proj, layer.k_proj, layer.v_proj]
    return [layer]


def _pnames(leaf):
    names = [n for n in ("mw", "Sw", "mb", "Sb") if getattr(leaf, n, None) is not None]
    if hasattr(leaf, "running_mean"):
        names += ["running_mean", "running_var"]
    return names


@pytest.mark.parametrize("cin,cout,stride,N,H", [(64, 64, 1, 16, 16), (64, 128, 2, 16, 16),
                                                 (8, 8, 1, 4, 8), (8, 16, 2, 4, 8)])
def test_resblock_layer(cin, cout, stride, N, H):
    kw = dict(gain_w=0.1, gain_b=0.1)
    dev, r32, r64 = _triple(lambda: ON.ResBlock(cin, cout, stride, **kw),
                            lambda: TT.ResBlock(cin, cout, stride, device=DEV, **kw))
    g = torch.Generator().manual_seed(cin + cout + stride)
    ma = torch.randn(N, cin, H, H, generator=g)
    Sa = torch.rand(N, cin, H, H, generator=g) * 0.1 + 1e-4
    Ho = H // stride
    dm = torch.randn(N, cout, Ho, Ho, generator=g) * 0.1
    dS = -torch.rand(N, cout, Ho, Ho, generator=g) * 1e-2
    _layer_step(dev, r32, r64, ma, Sa, dm, dS, F.get_cap_factor(N))


@pytest.mark.parametrize("B,S,E,H", [(4, 64, 128, 4), (2, 512, 512, 8)])
def test_mha_layer(B, S, E, H):
    dev, r32, r64 = _triple(lambda: ON.MultiheadAttentionV2(E, H, S),
                            lambda: TT.MultiheadAttentionV2(E, H, S, device=DEV))
    g = torch.Generator().manual_seed(B * S + E)
    ma = torch.randn(B, S, E, generator=g)
    Sa = torch.rand(B, S, E, generator=g) * 0.1
    dm = torch.randn(B, S, E, generator=g) * 0.1
    dS = -torch.rand(B, S, E, generator=g) * 1e-2
    _layer_step(dev, r32, r64, ma, Sa, dm, dS, F.get_cap_factor(B))
    # attention score rows are probability vectors with positive variances
    mu, var = dev.get_attention_scores()
    assert torch.allclose(mu.sum(-1), torch.ones_like(mu.sum(-1)), atol=1e-5)
    assert (var > 0).all()


def test_mha_zero_deltas_leave_parameters():
    """tests/validation/test_attention.py:445-464: zero deltas, unchanged weights."""
    E, H, S, B = 64, 4, 16, 2
    mha = TT.MultiheadAttentionV2(E, H, S, device=DEV)
    before = [t.clone() for t in params([mha])]
    ma = torch.randn(B, S, E, device=DEV)
    mha.forward(ma, torch.zeros_like(ma))
    z = torch.zeros(B, S, E, device=DEV)
    d_m, d_S = mha.backward(z, z)
    mha.update(F.get_cap_factor(B))
    assert torch.count_nonzero(d_m) == 0 and torch.count_nonzero(d_S) == 0
    for a, b in zip(before, params([mha])):
        assert torch.equal(a, b)


@pytest.mark.parametrize("cin,cout,k,stride,N,H", [
    (64, 64, 3, 1, 8, 32),     # transposed patches, bias row inside the contraction
    (256, 256, 3, 1, 16, 8),   # 2304 weight rows: the bias computed apart
    (64, 128, 2, 2, 8, 16),    # 2x2 stride-2 projection (256 weight rows)
    (3, 64, 3, 1, 4, 32),      # few weight rows
])
def test_conv_bias_sums_from_batchnorm(cin, cout, k, stride, N, H):
    """Conv → ReLU → BatchNorm as a container runs it: the BatchNorm backward
    sums its outgoing deltas per channel (tagi_bn_backward delta_sums) and the
    convolution takes its bias sums from them (tagi_param_grad_bias_given).
    The sums equal float64 sums of the deltas, and every parameter delta equals
    that of the convolution's own backward (bias sums computed by itself)."""
    from triton_tagi._chain import backward_chain

    torch.manual_seed(cin + cout + k)
    pad = 1 if k == 3 else 0
    conv = TT.Conv2D(cin, cout, k, stride=stride, padding=pad, device=DEV)
    relu, bn = TT.ReLU(), TT.BatchNorm2D(cout, device=DEV)
    twin = TT.Conv2D(cin, cout, k, stride=stride, padding=pad, device=DEV)
    for a, b in zip(params([twin]), params([conv])):
        a.copy_(b)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(N, cin, H, H, generator=g).to(DEV)
    Sx = (torch.rand(N, cin, H, H, generator=g) * 0.1).to(DEV)
    mz, Sz = conv.forward(x, Sx)
    twin.forward(x, Sx)
    ma, Sa = relu.forward(mz, Sz)
    bn.forward(ma, Sa)
    dm = (torch.randn(mz.shape, generator=g) * 0.1).to(DEV)
    dS = (-torch.rand(mz.shape, generator=g) * 1e-2).to(DEV)
    d_in = backward_chain([conv, relu, bn], dm, dS)
    # the deltas the convolution received: the BatchNorm+ReLU backward again
    dmz, dSz = bn.backward(dm, dS, relu=relu, delta_sums=True)
    sums = bn.delta_sums.cpu()
    want = torch.cat([dmz.double().sum((0, 2, 3)), dSz.double().sum((0, 2, 3))]).cpu()
    assert torch.allclose(sums, want, rtol=1e-9, atol=1e-12 * want.abs().max())
    d_twin = twin.backward(dmz, dSz)
    for a, b in zip(d_in, d_twin):
        assert torch.equal(a, b)
    for name in ("delta_mw", "delta_Sw", "delta_mb", "delta_Sb"):
        got, ref = getattr(conv, name), getattr(twin, name)
        err = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
        assert err <= 1e-6, (name, err)
