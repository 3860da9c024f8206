"""Generate golden vectors by running the reference implementation itself.

Run in a container where the triton-tagi sources are available (read-only):

    python tests/golden/make_golden.py /path/to/triton-tagi

It imports the reference package from that path with ``TRITON_INTERPRET=1``
(Triton kernels execute on the CPU; the three autotuned kernels are pinned to
one config so no GPU benchmarker is needed), runs seeded small cases of every
function on the hot path plus short ``Sequential.step`` trajectories, and
writes ``tests/golden/*.npz``. The GPU box never runs this script; tests only
read the committed ``.npz`` files.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def _setup(ref_root: str):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch  # noqa: F401
    import triton_tagi  # noqa: F401
    from triton_tagi.kernels import common

    for k in (common._fused_var_forward_kernel, common._fused_backward_delta_kernel,
              common._fused_weight_grad_kernel):
        k.configs = [k.configs[0]]


def _np(t):
    return t.detach().cpu().numpy().astype(np.float32)


def kernels():
    import torch
    from triton_tagi.kernels.attention import bmm_shared_left, bmm_shared_right, bmm_tagi_var
    from triton_tagi.kernels.common import (triton_fused_backward_delta, triton_fused_var_forward,
                                            triton_fused_weight_grad)
    from triton_tagi.layers.conv2d import _triton_col2im, _triton_im2col
    from triton_tagi.layers.relu import bayesian_relu
    from triton_tagi.layers.remax import triton_remax
    from triton_tagi.update.observation import compute_innovation
    from triton_tagi.update.parameters import update_parameters

    out = {}
    g = torch.Generator().manual_seed(1234)
    for tag, (M, K, N) in {"a": (37, 27, 10), "b": (64, 128, 96), "c": (5, 300, 33)}.items():
        ma = torch.randn(M, K, generator=g)
        Sa = torch.rand(M, K, generator=g) * 1e-2 + 1e-4
        mw = torch.randn(K, N, generator=g) / K**0.5
        Sw = torch.rand(K, N, generator=g) / K
        Sb = torch.rand(1, N, generator=g) * 1e-3
        dmz = torch.randn(M, N, generator=g) * 0.1
        dSz = -torch.rand(M, N, generator=g) * 1e-2
        out.update({f"gemm_{tag}_{k}": _np(v) for k, v in
                    dict(ma=ma, Sa=Sa, mw=mw, Sw=Sw, Sb=Sb, dmz=dmz, dSz=dSz).items()})
        out[f"gemm_{tag}_Sz"] = _np(triton_fused_var_forward(ma, Sa, mw, Sw, Sb))
        d_ma, d_Sa = triton_fused_backward_delta(dmz, dSz, mw)
        out[f"gemm_{tag}_d_ma"], out[f"gemm_{tag}_d_Sa"] = _np(d_ma), _np(d_Sa)
        gmw, gSw = triton_fused_weight_grad(ma, dmz, dSz)
        out[f"gemm_{tag}_gmw"], out[f"gemm_{tag}_gSw"] = _np(gmw), _np(gSw)

    # capped update: mixed signs, zero deltas, floor flips, three cap values
    n = 2000
    m = torch.randn(n, generator=g)
    S = torch.rand(n, generator=g) * 1e-2 + 1e-6
    dm = torch.randn(n, generator=g) * 0.05
    dS = torch.randn(n, generator=g) * 0.02
    dm[:50] = 0.0
    dS[50:100] = 0.0
    dS[100:200] = -10.0  # forces S' <= 0 → floor
    S[200:220] = 0.0     # exercises max(S, 1e-10)
    out.update(upd_m=_np(m), upd_S=_np(S), upd_dm=_np(dm), upd_dS=_np(dS))
    for cap in (0.1, 2.0, 3.0):
        mm, SS = m.clone(), S.clone()
        update_parameters(mm, SS, dm, dS, cap)
        out[f"upd_cap{cap}_m"], out[f"upd_cap{cap}_S"] = _np(mm), _np(SS)

    y = torch.randn(16, 10, generator=g)
    mu = torch.randn(16, 10, generator=g)
    var = torch.rand(16, 10, generator=g)
    dmu, dvar = compute_innovation(y, mu, var, 0.05)
    out.update(inn_y=_np(y), inn_mu=_np(mu), inn_var=_np(var), inn_dmu=_np(dmu),
               inn_dvar=_np(dvar))

    mz = torch.linspace(-8, 8, 4096)[torch.randperm(4096, generator=g)]
    Sz = torch.exp(torch.empty(4096).uniform_(-9, 1.5, generator=g))
    Sz[:16] = 0.0
    ma, Sa, J = bayesian_relu(mz, Sz)
    out.update(relu_mz=_np(mz), relu_Sz=_np(Sz), relu_ma=_np(ma), relu_Sa=_np(Sa), relu_J=_np(J))

    for tag, (B, K) in {"k10": (33, 10), "k64": (8, 64), "k512": (3, 512)}.items():
        mz = torch.randn(B, K, generator=g) * 2
        Sz = torch.rand(B, K, generator=g) * 2 + 1e-3
        ma, Sa, J = triton_remax(mz, Sz)
        out.update({f"remax_{tag}_{k}": _np(v) for k, v in
                    dict(mz=mz, Sz=Sz, ma=ma, Sa=Sa, J=J).items()})

    # attention products, including transposed (strided) operand views
    ma = torch.randn(2, 3, 17, 9, generator=g)
    va = torch.rand(2, 3, 17, 9, generator=g)
    mb = torch.randn(2, 3, 13, 9, generator=g)
    vb = torch.rand(2, 3, 13, 9, generator=g)
    out.update(att_ma=_np(ma), att_va=_np(va), att_mb=_np(mb), att_vb=_np(vb))
    out["att_var_t"] = _np(bmm_tagi_var(ma, va, mb.transpose(-1, -2), vb.transpose(-1, -2), 0.25))
    mR, vR = bmm_shared_right(ma, va, mb.transpose(-1, -2), scale=0.5)
    out["att_right_m"], out["att_right_v"] = _np(mR), _np(vR)
    bm = torch.randn(2, 3, 9, 11, generator=g)
    bv = torch.rand(2, 3, 9, 11, generator=g)
    out.update(att_bm=_np(bm), att_bv=_np(bv))
    mL, vL = bmm_shared_left(ma, bm, bv, scale=0.5)
    out["att_left_m"], out["att_left_v"] = _np(mL), _np(vL)

    # im2col / col2im with the reference's private helpers
    x = torch.randn(2, 3, 9, 7, generator=g)
    for tag, (k, s, p) in {"k3s1p1": (3, 1, 1), "k3s2p1": (3, 2, 1), "k2s2p0": (2, 2, 0),
                           "k5s1p2": (5, 1, 2)}.items():
        cols = _triton_im2col(x, k, k, s, p)
        out[f"im2col_{tag}"] = _np(cols)
        out[f"col2im_{tag}"] = _np(_triton_col2im(cols * 0.5 + 1.0, 2, 3, 9, 7, k, k, s, p))
    out["im2col_x"] = _np(x)
    np.savez_compressed(OUT / "kernels.npz", **out)


def _params(layers):
    """Flatten learnable parameters in a fixed order."""
    from triton_tagi.layers import BatchNorm2D, MultiheadAttentionV2, ResBlock

    seq = []
    for layer in layers:
        if isinstance(layer, ResBlock):
            seq += layer._learnable
        elif isinstance(layer, MultiheadAttentionV2):
            seq += [layer.q_proj, layer.k_proj, layer.v_proj]
        elif hasattr(layer, "mw") and layer.mw is not None:
            seq.append(layer)
    out = []
    for layer in seq:
        for name in ("mw", "Sw", "mb", "Sb"):
            t = getattr(layer, name, None)
            if t is not None:
                out.append(t)
        if isinstance(layer, BatchNorm2D):
            out += [layer.running_mean, layer.running_var]
    return out


def trajectories():
    import torch
    from triton_tagi import (AvgPool2D, BatchNorm2D, Conv2D, Embedding, Flatten, Linear,
                             MultiheadAttentionV2, PositionalEncoding, ReLU, Remax, ResBlock,
                             RMSNorm, Sequential)

    dev = "cpu"
    nets = {}

    torch.manual_seed(7)
    nets["mlp"] = (Sequential([Linear(784, 64, device=dev), ReLU(), Linear(64, 32, device=dev),
                               ReLU(), Linear(32, 10, device=dev), Remax()], device=dev),
                   torch.randn(16, 784), 10, 3)

    torch.manual_seed(8)
    nets["cnn"] = (Sequential([
        Conv2D(3, 8, 5, padding=2, device=dev), ReLU(), AvgPool2D(2),
        Conv2D(8, 16, 5, padding=2, device=dev), BatchNorm2D(16, device=dev), ReLU(),
        AvgPool2D(2),
        Flatten(), Linear(16 * 4 * 4, 32, device=dev), ReLU(), Linear(32, 10, device=dev),
        Remax()], device=dev), torch.randn(4, 3, 16, 16), 10, 2)

    torch.manual_seed(9)
    kw = dict(device=dev, gain_w=0.1, gain_b=0.1)
    nets["res"] = (Sequential([
        Conv2D(3, 8, 3, stride=1, padding=1, **kw), ReLU(), BatchNorm2D(8, **kw),
        ResBlock(8, 8, stride=1, **kw), ResBlock(8, 16, stride=2, **kw),
        AvgPool2D(4), Flatten(), Linear(16, 10, **kw), Remax()], device=dev),
        torch.randn(4, 3, 8, 8), 10, 2)

    torch.manual_seed(10)
    V, E, H, S = 16, 32, 4, 8
    nets["tfm"] = (Sequential([
        Embedding(V, E, input_size=S, scale=0.25, device=dev), PositionalEncoding(E, device=dev),
        MultiheadAttentionV2(E, H, S, bias=False, device=dev), RMSNorm(E, device=dev),
        Linear(E, 64, device=dev), ReLU(), Linear(64, E, device=dev), Linear(E, V, device=dev)],
        device=dev), torch.randint(0, V, (2, S)).float(), V, 2)

    for name, (net, x, n_cls, steps) in nets.items():
        out = {"x": _np(x)}
        g = torch.Generator().manual_seed(99)
        if name == "tfm":
            labels = torch.flip(x.long(), dims=[1])
            y = torch.nn.functional.one_hot(labels, n_cls).float()
        else:
            labels = torch.randint(0, n_cls, (x.shape[0],), generator=g)
            y = torch.nn.functional.one_hot(labels, n_cls).float()
        out["y"] = _np(y)
        for i, p in enumerate(_params(net.layers)):
            out[f"p0_{i:03d}"] = _np(p)
        for s in range(steps):
            mu, var = net.step(x, y, 0.05)
            out[f"mu_{s}"], out[f"var_{s}"] = _np(mu), _np(var)
        for i, p in enumerate(_params(net.layers)):
            out[f"p{steps}_{i:03d}"] = _np(p)
        out["steps"] = np.array(steps)
        np.savez_compressed(OUT / f"traj_{name}.npz", **out)
        print(name, "done", flush=True)


if __name__ == "__main__":
    _setup(sys.argv[1] if len(sys.argv) > 1 else "../triton-tagi")
    kernels()
    print("kernels done", flush=True)
    trajectories()
