"""Bayesian ReLU (drop-in for triton_tagi/layers/relu.py).

Moments of a = max(0, z), z ~ N(μ_z, S_z), with α = μ_z/σ_z (relu.py:63-86):
    μ_a = σ_z φ(α) + μ_z Φ(α)
    S_a = max(−μ_a² + 2μ_a μ_z − μ_z σ_z φ(α) + (S_z − μ_z²) Φ(α), 0)
    J   = Φ(α), with Φ(α) ≈ φ(α)/|α| for α < −5
Backward: δμ·J, δS·J².
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream
from ..base import Layer


def bayesian_relu(mz: Tensor, Sz: Tensor):
    """(ma, Sa, J) for any shape, processed flat (relu.py:94-122)."""
    check_cuda_f32(mz, Sz)
    mz, Sz = mz.contiguous(), Sz.contiguous()
    ma = torch.empty_like(mz)
    Sa = torch.empty_like(Sz)
    J = torch.empty_like(mz)
    lib()("tagi_relu_forward", mz.data_ptr(), Sz.data_ptr(), ma.data_ptr(), Sa.data_ptr(),
          J.data_ptr(), mz.numel(), stream(mz))
    return ma, Sa, J


def jacobian_backward(dm: Tensor, dS: Tensor, J: Tensor) -> tuple[Tensor, Tensor]:
    """(δμ·J, δS·J²) in one pass."""
    check_cuda_f32(dm, dS, J)
    dm, dS = dm.contiguous(), dS.contiguous()
    if dm.numel() != J.numel():
        raise ValueError("delta and Jacobian sizes differ")
    om = torch.empty_like(dm)
    oS = torch.empty_like(dS)
    lib()("tagi_jacobian_backward", dm.data_ptr(), dS.data_ptr(), J.data_ptr(), om.data_ptr(),
          oS.data_ptr(), dm.numel(), stream(dm))
    return om, oS


class ReLU(Layer):
    def __init__(self) -> None:
        self.J = None

    def forward(self, mz: Tensor, Sz: Tensor) -> tuple[Tensor, Tensor]:
        ma, Sa, J = bayesian_relu(mz, Sz)
        self.J = J.view(mz.shape)
        return ma.view(mz.shape), Sa.view(mz.shape)

    def backward(self, delta_mz: Tensor, delta_Sz: Tensor) -> tuple[Tensor, Tensor]:
        return jacobian_backward(delta_mz, delta_Sz, self.J)

    def __repr__(self):
        return "ReLU()"
