"""Fused moment contractions behind Linear and Conv2D.

Drop-in for triton_tagi/kernels/common.py: same function names, argument
meaning and return values, computed by libtagi_b200 (sm_100a CUDA).

    Sz      = ma² @ Sw + Sa @ (mw² + Sw) + Sb          (common.py:170-210)
    d_ma    = dmz @ mwᵀ,  d_Sa = dSz @ (mw²)ᵀ            (common.py:287-327)
    grad_mw = aᵀ @ dmz,   grad_Sw = (a²)ᵀ @ dSz          (common.py:410-451)
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream, workspace


def triton_fused_var_forward(ma: Tensor, Sa: Tensor, mw: Tensor, Sw: Tensor, Sb: Tensor) -> Tensor:
    """Sz (M, N) = ma² @ Sw + Sa @ (mw² + Sw) + Sb.

    ma, Sa: (M, K) with equal strides; mw, Sw: (K, N) with equal strides;
    Sb: (1, N) or (N,). Returns a new contiguous (M, N) tensor.
    """
    check_cuda_f32(ma, Sa, mw, Sw, Sb)
    M, K = ma.shape
    N = mw.shape[1]
    if Sa.stride() != ma.stride():
        ma, Sa = ma.contiguous(), Sa.contiguous()
    if Sw.stride() != mw.stride():
        mw, Sw = mw.contiguous(), Sw.contiguous()
    Sbv = Sb.reshape(-1).contiguous()
    Sz = torch.empty(M, N, device=ma.device, dtype=ma.dtype)
    lib()("tagi_fused_var_forward", ma.data_ptr(), Sa.data_ptr(), mw.data_ptr(), Sw.data_ptr(),
          Sbv.data_ptr(), Sz.data_ptr(), M, N, K, ma.stride(0), ma.stride(1), mw.stride(0),
          mw.stride(1), Sz.stride(0), Sz.stride(1), stream(ma))
    return Sz


def triton_fused_backward_delta(dmz: Tensor, dSz: Tensor, mw: Tensor) -> tuple[Tensor, Tensor]:
    """(d_ma, d_Sa), each (M, K): dmz @ mwᵀ and dSz @ (mw²)ᵀ."""
    check_cuda_f32(dmz, dSz, mw)
    if dSz.stride() != dmz.stride():
        dmz, dSz = dmz.contiguous(), dSz.contiguous()
    M, N = dmz.shape
    K = mw.shape[0]
    d_ma = torch.empty(M, K, device=dmz.device, dtype=dmz.dtype)
    d_Sa = torch.empty(M, K, device=dmz.device, dtype=dmz.dtype)
    lib()("tagi_fused_backward_delta", dmz.data_ptr(), dSz.data_ptr(), mw.data_ptr(),
          d_ma.data_ptr(), d_Sa.data_ptr(), M, K, N, dmz.stride(0), dmz.stride(1), mw.stride(0),
          mw.stride(1), d_ma.stride(0), d_ma.stride(1), stream(dmz))
    return d_ma, d_Sa


def triton_fused_weight_grad(a: Tensor, dmz: Tensor, dSz: Tensor) -> tuple[Tensor, Tensor]:
    """(grad_mw, grad_Sw), each (K, N): aᵀ @ dmz and (a²)ᵀ @ dSz."""
    check_cuda_f32(a, dmz, dSz)
    if dSz.stride() != dmz.stride():
        dmz, dSz = dmz.contiguous(), dSz.contiguous()
    M, K = a.shape
    N = dmz.shape[1]
    gmw = torch.empty(K, N, device=a.device, dtype=a.dtype)
    gSw = torch.empty(K, N, device=a.device, dtype=a.dtype)
    L = lib()
    hold, wp, wn = workspace(L.size("tagi_fused_weight_grad_workspace_size", M, K, N), a)
    L("tagi_fused_weight_grad", a.data_ptr(), dmz.data_ptr(), dSz.data_ptr(), gmw.data_ptr(),
      gSw.data_ptr(), M, K, N, a.stride(0), a.stride(1), dmz.stride(0), dmz.stride(1),
      gmw.stride(0), gmw.stride(1), wp, wn, stream(a))
    del hold
    return gmw, gSw
