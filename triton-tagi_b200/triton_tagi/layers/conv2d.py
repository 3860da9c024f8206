"""Bayesian Conv2D via patches (drop-in for triton_tagi/layers/conv2d.py).

Forward (conv2d.py:254-309): the fused moment contraction
    μ_z = P_μ @ μ_w + μ_b,  S_z = P_μ² @ S_w + P_S @ (μ_w² + S_w) + S_b
over the patches P (N·L, C·k·k) gathers them from the NCHW input itself (no
patch matrix in memory) and writes the result directly in NCHW.
Backward (conv2d.py:314-371): the reference forms the patch-space deltas
δP = δμ_z @ μ_wᵀ, δP_S = δS_z @ (μ_w²)ᵀ and folds them back to the input with
its col2im gather. For stride 1 one contraction over (tap, output channel) sums
the same terms: for each input pixel and tap it gathers the deltas at the output
position the col2im gather maps to (tagi_conv2d_backward_delta), so no
patch-space deltas exist in memory. For stride s > 1 only about 1/s² of the
(pixel, tap) pairs contribute, so the patch-space product and the gather
(tagi_backward_delta_view, tagi_col2im) do fewer flops and stay. The weight sums P_μᵀ·δμ_z, (P_μ²)ᵀ·δS_z
(bias as a row of ones) feed the parameter mode of the layer; the mean patches
are made for them from the input kept by forward.

``col2im_mode``: "reference" (default) gathers exactly as the reference's
_col2im_kernel (conv2d.py:119-130), which for stride > 1 does not test the
column offset for divisibility by the stride; "adjoint" is the true adjoint
of im2col. The two agree for stride 1.
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream, workspace
from ..base import LearnableLayer
from ..param_init import init_weight_bias_conv2d
from ._params import contiguous_params, weight_apply_sums, weight_param_backward, weight_update

_COL2IM_MODES = {"reference": 0, "adjoint": 1}


def _channels_last(xm: Tensor, xS: Tensor) -> tuple[Tensor, Tensor]:
    """NHWC copies of an NCHW tensor pair (tagi_nchw_to_nhwc)."""
    N, C, H, W = xm.shape
    ym = torch.empty(N, H, W, C, device=xm.device)
    yS = torch.empty_like(ym)
    lib()("tagi_nchw_to_nhwc", xm.data_ptr(), xS.data_ptr(), ym.data_ptr(), yS.data_ptr(), N, C,
          H * W, stream(xm))
    return ym, yS


class Conv2D(LearnableLayer):
    def __init__(self, C_in: int, C_out: int, kernel_size: int, stride: int = 1,
                 padding: int = 0, padding_type: int = 1, device="cuda", init_method="He",
                 gain_w: float = 1.0, gain_b: float = 1.0, col2im_mode: str = "reference") -> None:
        if padding_type not in (1, 2):
            raise ValueError("padding_type must be 1 (symmetric) or 2 (right/bottom)")
        if col2im_mode not in _COL2IM_MODES:
            raise ValueError(f"col2im_mode must be one of {sorted(_COL2IM_MODES)}")
        self.C_in, self.C_out = C_in, C_out
        self.kH = self.kW = kernel_size
        self.stride, self.padding, self.padding_type = stride, padding, padding_type
        self.col2im_mode = col2im_mode
        self.device = torch.device(device)
        self.mw, self.Sw, self.mb, self.Sb = init_weight_bias_conv2d(
            kernel_size, C_in, C_out, init_method=init_method, gain_w=gain_w, gain_b=gain_b,
            device=self.device)
        self.has_bias = True
        self.input_ma = None
        self.input_shape = None
        self.spatial = None
        self.delta_mw = self.delta_Sw = self.delta_mb = self.delta_Sb = None

    def _out_hw(self, H: int, W: int) -> tuple[int, int]:
        k, s, p = self.kH, self.stride, self.padding
        if self.padding_type == 2 and p > 0:
            return (H + p - k) // s + 1, (W + p - k) // s + 1
        return (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1

    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        check_cuda_f32(ma, Sa)
        contiguous_params(self)
        ma, Sa = ma.contiguous(), Sa.contiguous()
        N, C, H, W = ma.shape
        if C != self.C_in:
            raise ValueError(f"Conv2D expects {self.C_in} input channels, got {C}")
        self.input_shape = (N, C, H, W)
        Ho, Wo = self._out_hw(H, W)
        self.spatial = (Ho, Wo)
        Co = self.C_out
        dev = ma.device
        self.input_ma = ma  # the weight sums of backward take their patches from it
        mz = torch.empty(N, Co, Ho, Wo, device=dev)
        Sz = torch.empty(N, Co, Ho, Wo, device=dev)
        lb = lib()
        hold, wp, wn = workspace(
            lb.size("tagi_store_workspace_size", N * Ho * Wo, Co, C * self.kH * self.kW), ma)
        # channels-last copy of the input: the contraction then loads a tap's 8
        # channels with one 32-byte access instead of 8 plane-strided ones
        xm, xS = _channels_last(ma, Sa) if C % 8 == 0 else (ma, Sa)
        lb("tagi_conv2d_forward", xm.data_ptr(), xS.data_ptr(), self.mw.data_ptr(),
           self.Sw.data_ptr(), self.mb.data_ptr(), self.Sb.data_ptr(), mz.data_ptr(),
           Sz.data_ptr(), N, C, H, W, Co, self.kH, self.stride, self.padding,
           self.padding_type, 1 if C % 8 == 0 else 0, wp, wn, stream(ma))
        return mz, Sz

    def backward(self, delta_mz: Tensor, delta_Sz: Tensor,
                 bias_sums: Tensor | None = None) -> tuple[Tensor, Tensor]:
        """Input deltas and the parameter side. ``bias_sums``: the per-channel
        sums of (delta_mz, delta_Sz) when a container already has them (float64,
        2·C_out values, e.g. from the BatchNorm backward that produced the
        deltas); the bias then needs no pass over the deltas of its own."""
        check_cuda_f32(delta_mz, delta_Sz)
        dmz, dSz = delta_mz.contiguous(), delta_Sz.contiguous()
        N, C, H, W = self.input_shape
        Ho, Wo = self.spatial
        L, K, Co = Ho * Wo, C * self.kH * self.kW, self.C_out
        dev = dmz.device
        st = stream(dmz)
        d_map = (L, Co * L, 1, L)  # NCHW delta read as an (N·L) x Co matrix
        k, p = self.kH, self.padding
        d_ma = d_Sa = None
        if not self._skip_input_delta:
            d_ma = torch.empty(N, C, H, W, device=dev)
            d_Sa = torch.empty(N, C, H, W, device=dev)
            if self.stride == 1:
                # One contraction over (tap, co) gathers the deltas as the col2im fold
                # does (no patch-space deltas in memory).
                lb = lib()
                hold, wp, wn = workspace(
                    lb.size("tagi_store_workspace_size", N * H * W, C, Co * k * k), dmz)
                gm, gS = _channels_last(dmz, dSz) if Co % 8 == 0 else (dmz, dSz)
                lb("tagi_conv2d_backward_delta", gm.data_ptr(), gS.data_ptr(),
                   self.mw.data_ptr(), d_ma.data_ptr(), d_Sa.data_ptr(), N, C, H, W, Co, k, 1,
                   p, self.padding_type, _COL2IM_MODES[self.col2im_mode],
                   1 if Co % 8 == 0 else 0, wp, wn, st)
            else:
                # With stride s only about 1/s² of the (pixel, tap) pairs contribute:
                # the patch-space product plus the gather does the fewer flops.
                dpm = torch.empty(N * L, K, device=dev)
                dpS = torch.empty(N * L, K, device=dev)
                lib()("tagi_backward_delta_view", dmz.data_ptr(), dSz.data_ptr(), *d_map,
                      self.mw.data_ptr(), Co, dpm.data_ptr(), dpS.data_ptr(), 0, 0, K, 1, N * L,
                      K, Co, st)
                lib()("tagi_col2im", dpm.data_ptr(), dpS.data_ptr(), d_ma.data_ptr(),
                      d_Sa.data_ptr(), N, C, H, W, k, self.stride, p, self.padding_type,
                      _COL2IM_MODES[self.col2im_mode], st)
                del dpm, dpS
        if Co <= 64 and (N * L) % 8 == 0:
            # Up to 64 output channels the weight-sum tiles stage each patch
            # column (c, kh, kw) as one thread's row: the transposed patches give
            # it contiguous pixels.
            pt = torch.empty(K, N * L, device=dev)
            lib()("tagi_im2col_t", self.input_ma.data_ptr(), pt.data_ptr(), N, C, H, W, k,
                  self.stride, p, self.padding_type, st)
            weight_param_backward(self, pt, N * L, (dmz, dSz), d_map, N * L, K, Co, True,
                                  transposed=True, bias_sums=bias_sums)
        else:
            pm = torch.empty(N * L, K, device=dev)
            lib()("tagi_im2col", self.input_ma.data_ptr(), None, pm.data_ptr(), None, N, C, H,
                  W, k, self.stride, p, self.padding_type, st)
            weight_param_backward(self, pm, K, (dmz, dSz), d_map, N * L, K, Co, True,
                                  bias_sums=bias_sums)
        return d_ma, d_Sa

    def update(self, cap_factor: float) -> None:
        weight_update(self, cap_factor, True)

    def _sums_numel(self) -> int:
        return 2 * (self.C_in * self.kH * self.kW + 1) * self.C_out

    def _apply_sums(self, buf: Tensor, cap: float) -> None:
        weight_apply_sums(self, buf, self.C_in * self.kH * self.kW, self.C_out, True, cap)

    @property
    def num_parameters(self) -> int:
        return 2 * (self.mw.numel() + self.mb.numel())

    def __repr__(self):
        return (f"Conv2D({self.C_in}, {self.C_out}, kernel={self.kH}, stride={self.stride}, "
                f"pad={self.padding})")
