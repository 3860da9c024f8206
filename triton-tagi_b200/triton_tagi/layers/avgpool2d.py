"""Bayesian average pooling (drop-in for triton_tagi/layers/avgpool2d.py).

Window = stride = k. μ_out = Σμ/k²; S_out = ΣS/k⁴ (independent pixels,
default) or ΣS/k² (``spatial_correlation=True``). Backward spreads each
window's deltas with the same scales (avgpool2d.py:92-130); pixels past the
last full window (H or W not divisible by k) receive zero.
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream
from ..base import Layer


class AvgPool2D(Layer):
    def __init__(self, kernel_size: int, spatial_correlation: bool = False) -> None:
        self.k = kernel_size
        self.spatial_correlation = spatial_correlation
        self.input_shape = None

    def _var_scale(self) -> float:
        inv_k2 = 1.0 / (self.k * self.k)
        return inv_k2 if self.spatial_correlation else inv_k2 * inv_k2

    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        check_cuda_f32(ma, Sa)
        ma, Sa = ma.contiguous(), Sa.contiguous()
        self.input_shape = ma.shape
        N, C, H, W = ma.shape
        k = self.k
        om = torch.empty(N, C, H // k, W // k, device=ma.device)
        oS = torch.empty_like(om)
        lib()("tagi_avgpool_forward", ma.data_ptr(), Sa.data_ptr(), om.data_ptr(), oS.data_ptr(),
              N, C, H, W, k, self._var_scale(), stream(ma))
        return om, oS

    def backward(self, dm: Tensor, ds: Tensor) -> tuple[Tensor, Tensor]:
        check_cuda_f32(dm, ds)
        dm, ds = dm.contiguous(), ds.contiguous()
        N, C, H, W = self.input_shape
        om = torch.empty(N, C, H, W, device=dm.device)
        oS = torch.empty_like(om)
        lib()("tagi_avgpool_backward", dm.data_ptr(), ds.data_ptr(), om.data_ptr(), oS.data_ptr(),
              N, C, H, W, self.k, self._var_scale(), stream(dm))
        return om, oS

    def __repr__(self):
        sc = "on" if self.spatial_correlation else "off"
        return f"AvgPool2D(kernel={self.k}, spatial_correlation={sc})"
