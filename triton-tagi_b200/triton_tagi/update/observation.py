"""Output innovation (drop-in for the dense path of triton_tagi/update/observation.py).

    δμ = (y − μ) / (S + σv²),   δS = −1 / (S + σv²)
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream


def compute_innovation(y: Tensor, y_pred_mu: Tensor, y_pred_var: Tensor, sigma_v: float):
    """Dense innovation (observation.py:119-163). The heteroscedastic branch
    (predictions twice as wide as y) is not part of this library."""
    if y_pred_mu.shape[-1] == 2 * y.shape[-1] and y.shape[-1] != 0:
        raise NotImplementedError("heteroscedastic (TAGI-V) innovation is not implemented")
    check_cuda_f32(y, y_pred_mu, y_pred_var)
    if y.shape != y_pred_mu.shape or y.shape != y_pred_var.shape:
        raise ValueError(f"shape mismatch: y {tuple(y.shape)} vs prediction {tuple(y_pred_mu.shape)}")
    y, mu, var = y.contiguous(), y_pred_mu.contiguous(), y_pred_var.contiguous()
    dmu = torch.empty_like(y)
    dvar = torch.empty_like(y)
    lib()("tagi_innovation", y.data_ptr(), mu.data_ptr(), var.data_ptr(), dmu.data_ptr(),
          dvar.data_ptr(), y.numel(), float(sigma_v) ** 2, stream(y))
    return dmu, dvar
