"""Bayesian RMSNorm (drop-in for triton_tagi/layers/rms_norm.py).

Per row over the feature dim (rms_norm.py:93-110):
    inv = 1/√(mean(μ_a² + S_a) + ε)
    μ_z = inv μ_a μ_γ,   S_z = inv² (S_a (μ_γ² + S_γ) + S_γ μ_a²)
Backward (rms_norm.py:115-128): δμ_a = inv μ_γ δμ_z, δS_a = (inv μ_γ)² δS_z;
γ sums Σ inv μ_a δμ_z and Σ inv² μ_a² δS_z over rows (float64).
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import WGRAD_DELTAS, WGRAD_UPDATE, check_cuda_f32, lib, stream
from ..base import LearnableLayer
from ..param_init import init_weight_bias_norm
from ._params import contiguous_params


class RMSNorm(LearnableLayer):
    def __init__(self, normalized_shape, eps: float = 1e-6, gain_w: float = 1.0,
                 device="cuda") -> None:
        if isinstance(normalized_shape, int):
            normalized_shape = [normalized_shape]
        if len(normalized_shape) != 1:
            raise ValueError(
                f"RMSNorm only supports a single normalized dimension, got {normalized_shape}")
        self.normalized_shape = list(normalized_shape)
        self.ni = normalized_shape[0]
        self.eps = eps
        self.gain_w = gain_w
        self.device = torch.device(device)
        self.has_bias = False
        self.mw, self.Sw, _, _ = init_weight_bias_norm(self.ni, gain_w=gain_w, gain_b=1.0,
                                                       device=self.device)
        self.mb = self.Sb = None
        self.ma_in = None
        self.inv_rms = None
        self._input_shape = None
        self.delta_mw = self.delta_Sw = self.delta_mb = self.delta_Sb = None

    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        check_cuda_f32(ma, Sa)
        contiguous_params(self, ("mw", "Sw"))
        self._input_shape = ma.shape
        a = ma.reshape(-1, self.ni).contiguous()
        s = Sa.reshape(-1, self.ni).contiguous()
        rows = a.shape[0]
        mz = torch.empty_like(a)
        Sz = torch.empty_like(a)
        inv = torch.empty(rows, 1, device=a.device)
        lib()("tagi_rmsnorm_forward", a.data_ptr(), s.data_ptr(), self.mw.data_ptr(),
              self.Sw.data_ptr(), mz.data_ptr(), Sz.data_ptr(), inv.data_ptr(), rows, self.ni,
              float(self.eps), stream(a))
        self.ma_in, self.inv_rms = a, inv
        return mz.reshape(self._input_shape), Sz.reshape(self._input_shape)

    def backward(self, delta_mz: Tensor, delta_Sz: Tensor) -> tuple[Tensor, Tensor]:
        check_cuda_f32(delta_mz, delta_Sz)
        shape = delta_mz.shape
        dm = delta_mz.reshape(-1, self.ni).contiguous()
        dS = delta_Sz.reshape(-1, self.ni).contiguous()
        rows = dm.shape[0]
        dma = torch.empty_like(dm)
        dSa = torch.empty_like(dS)
        mode = self._param_mode
        sums = (self._reducer.buffer(self, 2 * self.ni, torch.float64) if mode == "sums"
                else torch.empty(2 * self.ni, device=dm.device, dtype=torch.float64))
        st = stream(dm)
        L = lib()
        L("tagi_rmsnorm_backward", dm.data_ptr(), dS.data_ptr(), self.ma_in.data_ptr(),
          self.inv_rms.data_ptr(), self.mw.data_ptr(), dma.data_ptr(), dSa.data_ptr(),
          sums.data_ptr(), rows, self.ni, st)
        if mode == "deltas":
            self.delta_mw = torch.empty(self.ni, device=dm.device)
            self.delta_Sw = torch.empty(self.ni, device=dm.device)
            L("tagi_apply_vector_sums", sums.data_ptr(), sums[self.ni:].data_ptr(), self.ni,
              WGRAD_DELTAS, None, self.Sw.data_ptr(), self.delta_mw.data_ptr(),
              self.delta_Sw.data_ptr(), 1.0, st)
        elif mode == "update":
            self._apply_sums(sums, self._cap)
            self._updated_in_backward = True
        elif mode == "sums":
            self._reducer.ready(self)
        else:
            raise ValueError(f"unknown parameter mode {mode!r}")
        return dma.reshape(shape), dSa.reshape(shape)

    def _sums_numel(self) -> int:
        return 2 * self.ni

    def _apply_sums(self, sums: Tensor, cap: float) -> None:
        lib()("tagi_apply_vector_sums", sums.data_ptr(), sums[self.ni:].data_ptr(), self.ni,
              WGRAD_UPDATE, self.mw.data_ptr(), self.Sw.data_ptr(), None, None, float(cap),
              stream(sums))

    def update(self, cap_factor: float) -> None:
        from ..update.parameters import update_parameters

        if self._updated_in_backward:
            self._updated_in_backward = False
            return
        if self._param_mode == "sums":
            return
        update_parameters(self.mw, self.Sw, self.delta_mw, self.delta_Sw, cap_factor)

    @property
    def num_parameters(self) -> int:
        return 2 * self.mw.numel()

    def __repr__(self) -> str:
        return f"RMSNorm(normalized_shape={self.normalized_shape}, eps={self.eps}, gain_w={self.gain_w})"
