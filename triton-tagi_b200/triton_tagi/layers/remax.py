"""Remax (drop-in for triton_tagi/layers/remax.py).

Row-wise over the last dim (remax.py:33-114): MixtureReLU moments of
M = max(0, Z); log-normal moments of M and M̃ = ΣM; A = M/M̃ renormalised so
Σμ_A = 1; J = cov(A, Z)/var(Z) with cov(A, Z) = cov(A, M)/Φ(α) capped by the
Cauchy–Schwarz bound. The reference's log/exp closed form cancels (its own
float32 evaluation is off by up to ~1 relative in variance and Jacobian on
attention rows); tagi_remax_forward evaluates the same quantities through exact
rational forms without cancelling terms, in float32 with float64 row sums,
within a few 1e-6 of a float64 evaluation of the reference's formulas.
Backward: δμ·J, δS·J².
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream
from ..base import Layer
from .relu import jacobian_backward


def triton_remax(mu_z: Tensor, var_z: Tensor):
    """(mu_a, var_a, J) for (B, K) or (K,) inputs (remax.py:122-164)."""
    check_cuda_f32(mu_z, var_z)
    squeeze = mu_z.dim() == 1
    mz = mu_z.reshape(1, -1) if squeeze else mu_z.reshape(-1, mu_z.shape[-1])
    Sz = var_z.reshape(mz.shape)
    mz, Sz = mz.contiguous(), Sz.contiguous()
    B, K = mz.shape
    ma = torch.empty_like(mz)
    Sa = torch.empty_like(mz)
    J = torch.empty_like(mz)
    lib()("tagi_remax_forward", mz.data_ptr(), Sz.data_ptr(), ma.data_ptr(), Sa.data_ptr(),
          J.data_ptr(), B, K, K, stream(mz))
    shape = mu_z.shape
    return ma.reshape(shape), Sa.reshape(shape), J.reshape(shape)


class Remax(Layer):
    def __init__(self) -> None:
        self.J = None

    def forward(self, mz: Tensor, Sz: Tensor) -> tuple[Tensor, Tensor]:
        mu_a, Sa, J = triton_remax(mz, Sz)
        self.J = J
        return mu_a, Sa

    def backward(self, delta_ma: Tensor, delta_Sa: Tensor) -> tuple[Tensor, Tensor]:
        return jacobian_backward(delta_ma, delta_Sa, self.J)

    def __repr__(self) -> str:
        return "Remax()"
