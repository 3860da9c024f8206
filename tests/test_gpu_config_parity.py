"""Parity at the benchmark configurations, at the benchmark sizes, per layer.

* MLP (batch 256), CNN (batch 512), ResNet-18 (batch 128: the benchmark's cap
  factor and split plans) and the transformer at full width (E = 512, S = 512,
  8 heads, 4 blocks; batch 4): each ``Sequential.step`` runs on the GPU exactly
  as in the benchmark, and every layer is checked against the CPU oracle fed
  with that layer's own GPU inputs (teacher forcing, ``_teacher``): means
  normwise ≤ 1e-5, variances and variance deltas element-wise ≤ 1e-4,
  updated variances element-wise ≤ 1e-4 of the pre-update variance. Two steps
  where BatchNorm's running statistics move (their EMA starts on step 2).
* The Linear op sweep at every shape, the 8192 × 4096 ×
  4096 headline included: forward, input deltas and the weight sums with the
  fused capped update, against the float64 oracle on a random subset of rows
  (forward, input deltas: rows are independent) and columns (weight sums and
  update: columns are independent, each over the full batch reduction).

Run with ``-s`` (or ``-rP``) to see the per-layer tables.
"""

from __future__ import annotations

import pytest
import torch

import oracle.moments as F
import oracle.net as ON
import triton_tagi as TT
from _nets import build_config, copy_params
from _teacher import assert_report, teacher_forced_step
from _tol import MEAN_RTOL, VAR_RTOL, elem_check, rel_err, var_update_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(name, batch, seed):
    g = torch.Generator().manual_seed(seed)
    if name == "mlp":
        x = torch.randn(batch, 784, generator=g)
    elif name == "tfm":
        x = torch.randint(0, 64, (batch, 512), generator=g).float()
    else:
        x = torch.randn(batch, 3, 32, 32, generator=g)
    if name == "tfm":
        y = torch.nn.functional.one_hot(torch.flip(x.long(), dims=[1]), 64).float()
    else:
        y = torch.nn.functional.one_hot(torch.randint(0, 10, (batch,), generator=g), 10).float()
    return x, y


@pytest.mark.parametrize("name,batch,steps", [("mlp", 256, 2), ("cnn", 512, 2), ("r18", 128, 2),
                                              ("tfm", 4, 1)])
def test_config_per_layer_teacher_forced(name, batch, steps):
    torch.manual_seed(0)
    ref32 = build_config(name, ON)
    ref64 = build_config(name, ON)
    dev = build_config(name, TT, device=DEV)
    copy_params(ref32, dev, DEV)
    net = TT.Sequential(dev, device=DEV)
    for s in range(steps):
        x, y = _inputs(name, batch, 10 + s)
        rep = teacher_forced_step(net, ref32, ref64, x.to(DEV), y.to(DEV), 0.05,
                                  what=f"{name} batch {batch} step {s}")
        assert_report(rep)


SWEEP = [(m, k) for m in (8192, 4096, 1024, 256) for k in (4096, 1024)]


@pytest.mark.parametrize("M,K", SWEEP)
def test_linear_sweep_shape(M, K):
    """mu_a~N(0,1), var_a~U(1e-4,1e-2), mu_W~N(0,1/K),
    var_W=U(0.5,1.5)/K, mu_b=0, var_b=1e-3, delta_mu~N(0,1e-2),
    delta_var~-U(0,1e-2); forward, input deltas, weight sums + capped update."""
    N = K
    g = torch.Generator().manual_seed(M * 7 + K)
    ma = torch.randn(M, K, generator=g)
    Sa = torch.rand(M, K, generator=g) * (1e-2 - 1e-4) + 1e-4
    mw = torch.randn(K, N, generator=g) / K**0.5
    Sw = (torch.rand(K, N, generator=g) + 0.5) / K
    mb, Sb = torch.zeros(1, N), torch.full((1, N), 1e-3)
    dmz = torch.randn(M, N, generator=g) * 0.1
    dSz = -torch.rand(M, N, generator=g) * 1e-2
    rows = torch.randperm(M, generator=g)[:256].sort().values
    cols = torch.randperm(N, generator=g)[:256].sort().values

    lin = TT.Linear(K, N, device=DEV)
    lin.mw, lin.Sw, lin.mb, lin.Sb = (t.to(DEV) for t in (mw, Sw, mb, Sb))
    mz, Sz = lin.forward(ma.to(DEV), Sa.to(DEV))
    cap = F.get_cap_factor(M)
    lin._set_param_mode("update", cap)
    try:
        d_ma, d_Sa = lin.backward(dmz.to(DEV), dSz.to(DEV))
    finally:
        lin._set_param_mode("deltas")
    torch.cuda.synchronize()
    d = lambda t: t.double()  # noqa: E731

    # forward on the row subset
    ex_m = F.mean_forward(d(ma[rows]), d(mw), d(mb))
    ex_S = F.var_forward(d(ma[rows]), d(Sa[rows]), d(mw), d(Sw), d(Sb))
    assert rel_err(mz.cpu()[rows], ex_m) <= MEAN_RTOL, rel_err(mz.cpu()[rows], ex_m)
    w, _, e = elem_check(Sz.cpu()[rows], ex_S, ex_S, VAR_RTOL)
    assert w <= 1.0, f"forward variance: element-wise {e:.3e}"
    # input deltas (pre-update weights) on the row subset
    r_ma, r_Sa = F.backward_delta(d(dmz[rows]), d(dSz[rows]), d(mw))
    assert rel_err(d_ma.cpu()[rows], r_ma) <= MEAN_RTOL, rel_err(d_ma.cpu()[rows], r_ma)
    w, _, e = elem_check(d_Sa.cpu()[rows], r_Sa, r_Sa, VAR_RTOL)
    assert w <= 1.0, f"input variance deltas: element-wise {e:.3e}"
    # weight sums + capped update on the column subset (full reduction over M)
    gm, gS = F.weight_grad(d(ma), d(dmz[:, cols]), d(dSz[:, cols]))
    sw, sb = d(Sw[:, cols]), d(Sb[:, cols])
    ex_mw, ex_Sw = F.capped_update(d(mw[:, cols]), sw, sw * gm, sw * sw * gS, cap)
    ex_mb, ex_Sb = F.capped_update(d(mb[:, cols]), sb, sb * d(dmz[:, cols]).sum(0, keepdim=True),
                                   sb * sb * d(dSz[:, cols]).sum(0, keepdim=True), cap)
    got = {n: getattr(lin, n).cpu()[:, cols] for n in ("mw", "Sw", "mb", "Sb")}
    assert rel_err(got["mw"], ex_mw) <= MEAN_RTOL, rel_err(got["mw"], ex_mw)
    assert rel_err(got["mb"], ex_mb) <= MEAN_RTOL, rel_err(got["mb"], ex_mb)
    assert var_update_err(got["Sw"], ex_Sw, sw) <= VAR_RTOL, var_update_err(got["Sw"], ex_Sw, sw)
    assert var_update_err(got["Sb"], ex_Sb, sb) <= VAR_RTOL, var_update_err(got["Sb"], ex_Sb, sb)
    print(f"\nsweep {M}x{K}x{N}: forward mean {rel_err(mz.cpu()[rows], ex_m):.2e}, "
          f"input deltas mean {rel_err(d_ma.cpu()[rows], r_ma):.2e}, "
          f"updated mw {rel_err(got['mw'], ex_mw):.2e}, Sw {var_update_err(got['Sw'], ex_Sw, sw):.2e}")
    from triton_tagi._lib import device_status

    assert device_status(reset=True) == 0
