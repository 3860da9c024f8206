"""Bayesian fully-connected layer (drop-in for triton_tagi/layers/linear.py).

Forward (one fused kernel for mean and variance, linear.py:83-103):
    μ_z = μ_a @ μ_w + μ_b
    S_z = μ_a² @ S_w + S_a @ (μ_w² + S_w) + S_b
Backward (linear.py:108-156):
    δμ_a = δμ_z @ μ_wᵀ,  δS_a = δS_z @ (μ_w²)ᵀ      (pre-update weights)
    Δμ_w = S_w·(μ_aᵀ @ δμ_z),  ΔS_w = S_w²·((μ_a²)ᵀ @ δS_z),  bias likewise
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream, workspace
from ..base import LearnableLayer
from ..param_init import init_weight_bias_linear
from ._params import contiguous_params, weight_apply_sums, weight_param_backward, weight_update


class Linear(LearnableLayer):
    def __init__(self, in_features: int, out_features: int, device="cuda", init_method="He",
                 gain_w: float = 1.0, gain_b: float = 1.0, bias: bool = True) -> None:
        self.in_features = in_features
        self.out_features = out_features
        self.device = torch.device(device)
        self.has_bias = bias
        self.mw, self.Sw, self.mb, self.Sb = init_weight_bias_linear(
            in_features, out_features, init_method=init_method, gain_w=gain_w, gain_b=gain_b,
            bias=bias, device=self.device)
        self.ma_in = None
        self.delta_mw = self.delta_Sw = self.delta_mb = self.delta_Sb = None

    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        check_cuda_f32(ma, Sa)
        contiguous_params(self)
        K, N = self.in_features, self.out_features
        self._input_shape = ma.shape
        a = ma.reshape(-1, K).contiguous()
        s = Sa.reshape(-1, K).contiguous()
        self.ma_in = a
        M = a.shape[0]
        mz = torch.empty(M, N, device=a.device)
        Sz = torch.empty(M, N, device=a.device)
        L = lib()
        # small batches split the reduction over the idle SMs (workspace sized by the library)
        hold, wp, wn = workspace(L.size("tagi_store_workspace_size", M, N, K), a)
        L("tagi_linear_forward", a.data_ptr(), s.data_ptr(), self.mw.data_ptr(),
          self.Sw.data_ptr(), self.mb.data_ptr() if self.has_bias else None,
          self.Sb.data_ptr() if self.has_bias else None, mz.data_ptr(), Sz.data_ptr(), M, K, N,
          wp, wn, stream(a))
        out = (*self._input_shape[:-1], N)
        return mz.reshape(out), Sz.reshape(out)

    def backward(self, delta_mz: Tensor, delta_Sz: Tensor) -> tuple[Tensor, Tensor]:
        check_cuda_f32(delta_mz, delta_Sz)
        K, N = self.in_features, self.out_features
        dm = delta_mz.reshape(-1, N).contiguous()
        dS = delta_Sz.reshape(-1, N).contiguous()
        M = dm.shape[0]
        d_ma = d_Sa = None
        if not self._skip_input_delta:
            d_ma = torch.empty(M, K, device=dm.device)
            d_Sa = torch.empty(M, K, device=dm.device)
            L = lib()
            hold, wp, wn = workspace(L.size("tagi_store_workspace_size", M, K, N), dm)
            L("tagi_linear_backward_delta", dm.data_ptr(), dS.data_ptr(), self.mw.data_ptr(),
              d_ma.data_ptr(), d_Sa.data_ptr(), M, K, N, wp, wn, stream(dm))
        weight_param_backward(self, self.ma_in, K, (dm, dS), (0, 0, N, 1), M, K, N, self.has_bias)
        if d_ma is None:
            return None, None
        shp = (*self._input_shape[:-1], K)
        return d_ma.reshape(shp), d_Sa.reshape(shp)

    def update(self, cap_factor: float) -> None:
        weight_update(self, cap_factor, self.has_bias)

    def _sums_numel(self) -> int:
        return 2 * (self.in_features + (1 if self.has_bias else 0)) * self.out_features

    def _apply_sums(self, buf: Tensor, cap: float) -> None:
        weight_apply_sums(self, buf, self.in_features, self.out_features, self.has_bias, cap)

    @property
    def num_parameters(self) -> int:
        n = self.mw.numel() + (self.mb.numel() if self.has_bias else 0)
        return 2 * n

    def __repr__(self):
        return f"Linear(in={self.in_features}, out={self.out_features}, bias={self.has_bias})"
