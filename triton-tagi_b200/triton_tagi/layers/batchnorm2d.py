"""Bayesian BatchNorm2D (drop-in for triton_tagi/layers/batchnorm2d.py).

Training mode normalises with the batch statistics (batchnorm2d.py:386-396):
    mean_c = E[μ_z],  var_c = (E[S_z] + E[μ_z²] − mean_c²)·n/(n−1)
computed from one pass of float64 per-channel sums (the reference makes three
reduction launches and an μ_z² temporary). The first training call initialises
the running statistics (and γ = √(var+ε) when ``preserve_var``), later calls
update them with an exponential moving average (batchnorm2d.py:341-355).
Affine with Gaussian γ, β (batchnorm2d.py:59-126):
    μ̂ = (μ_z − mean)/√(var+ε),  Ŝ = S_z/(var+ε)
    μ_a = μ_γ μ̂ + μ_β,  S_a = μ_γ² Ŝ + S_γ μ̂² + S_γ Ŝ + S_β
Backward (batchnorm2d.py:436-513): δμ_z = δμ_a μ_γ/√(var+ε),
δS_z = δS_a μ_γ²/(var+ε), with the γ/β batch sums reduced in the same pass.

Under data parallelism the channel sums (forward) and γ/β sums (backward) are
all-reduced, so statistics and updates use the global batch.
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import WGRAD_DELTAS, WGRAD_UPDATE, check_cuda_f32, lib, stream
from ..base import LearnableLayer
from ..param_init import init_weight_bias_norm
from ._params import contiguous_params


class BatchNorm2D(LearnableLayer):
    def __init__(self, num_features: int, momentum: float = 0.1, eps: float = 1e-5,
                 device="cuda", gain_w: float = 1.0, gain_b: float = 1.0,
                 preserve_var: bool = True) -> None:
        self.num_features = num_features
        self.momentum = momentum
        self.eps = eps
        self.device = torch.device(device)
        self.training = True
        self.preserve_var = preserve_var
        self._is_initialized = False
        self.mw, self.Sw, self.mb, self.Sb = init_weight_bias_norm(
            num_features, gain_w=gain_w, gain_b=gain_b, device=self.device)
        self.has_bias = True
        self.running_mean = torch.zeros(num_features, device=self.device)
        self.running_var = torch.ones(num_features, device=self.device)
        self.m_hat = None
        self.S_hat = None
        self.input_shape = None
        self._norm_mean = None
        self._norm_var = None
        self.delta_mw = self.delta_Sw = self.delta_mb = self.delta_Sb = None
        # Data-parallel hook: a callable that all-reduces a float64 tensor in place.
        self._stats_allreduce = None
        self._stats_world = 1

    def train(self) -> None:
        self.training = True

    def eval(self) -> None:
        self.training = False

    def forward(self, mz: Tensor, Sz: Tensor, residual=None) -> tuple[Tensor, Tensor]:
        """Normalised moments; ``residual`` = (μ, S) of a stream to add to them
        (the ResBlock shortcut), as ``triton_add_shortcut`` after this layer."""
        check_cuda_f32(mz, Sz)
        contiguous_params(self, ("mw", "Sw", "mb", "Sb", "running_mean", "running_var"))
        mz, Sz = mz.contiguous(), Sz.contiguous()
        self.input_shape = mz.shape
        N, C, H, W = mz.shape
        HW = H * W
        dev = mz.device
        st = stream(mz)
        L = lib()
        if residual is not None:
            if residual[0].shape != mz.shape or residual[1].shape != mz.shape:
                raise ValueError("BatchNorm2D: residual shape differs from the output's")
            check_cuda_f32(*residual)
            residual = (residual[0].contiguous(), residual[1].contiguous())
        if self.training and self._stats_allreduce is None:
            # one launch: sums, statistics and normalisation per channel cluster
            mean = torch.empty(C, device=dev)
            var = torch.empty(C, device=dev)
            ma = torch.empty_like(mz)
            Sa = torch.empty_like(Sz)
            self.m_hat = torch.empty_like(mz)
            self.S_hat = None
            L("tagi_bn_train_forward", mz.data_ptr(), Sz.data_ptr(), mean.data_ptr(),
              var.data_ptr(), self.running_mean.data_ptr(), self.running_var.data_ptr(),
              self.mw.data_ptr(), self.Sw.data_ptr(), self.mb.data_ptr(), self.Sb.data_ptr(),
              ma.data_ptr(), Sa.data_ptr(), self.m_hat.data_ptr(),
              residual[0].data_ptr() if residual is not None else None,
              residual[1].data_ptr() if residual is not None else None, N, C, HW,
              0 if self._is_initialized else 1, 1 if self.preserve_var else 0,
              float(self.momentum), float(self.eps), st)
            self._is_initialized = True
            self._norm_mean, self._norm_var = mean, var
            return ma, Sa
        if self.training:
            # SyncBN: channel sums, all-reduced, then one launch that finalises
            # the statistics and normalises (residual added)
            sums = torch.empty(3 * C, device=dev, dtype=torch.float64)
            L("tagi_bn_channel_sums", mz.data_ptr(), Sz.data_ptr(), sums.data_ptr(), N, C, HW, st)
            self._stats_allreduce(sums)
            count = float(N * HW) * self._stats_world
            mean = torch.empty(C, device=dev)
            var = torch.empty(C, device=dev)
            ma = torch.empty_like(mz)
            Sa = torch.empty_like(Sz)
            self.m_hat = torch.empty_like(mz)
            self.S_hat = None
            L("tagi_bn_sync_forward", mz.data_ptr(), Sz.data_ptr(), sums.data_ptr(), count,
              mean.data_ptr(), var.data_ptr(), self.running_mean.data_ptr(),
              self.running_var.data_ptr(), self.mw.data_ptr(), self.Sw.data_ptr(),
              self.mb.data_ptr(), self.Sb.data_ptr(), ma.data_ptr(), Sa.data_ptr(),
              self.m_hat.data_ptr(), residual[0].data_ptr() if residual is not None else None,
              residual[1].data_ptr() if residual is not None else None, N, C, HW,
              0 if self._is_initialized else 1, 1 if self.preserve_var else 0,
              float(self.momentum), float(self.eps), st)
            self._is_initialized = True
            self._norm_mean, self._norm_var = mean, var
            return ma, Sa
        else:
            mean, var = self.running_mean, self.running_var
        self._norm_mean, self._norm_var = mean, var
        ma = torch.empty_like(mz)
        Sa = torch.empty_like(Sz)
        self.m_hat = torch.empty_like(mz)
        self.S_hat = None  # not needed by backward (the reference caches but never reads it)
        L("tagi_bn_forward", mz.data_ptr(), Sz.data_ptr(), mean.data_ptr(), var.data_ptr(),
          self.mw.data_ptr(), self.Sw.data_ptr(), self.mb.data_ptr(), self.Sb.data_ptr(),
          ma.data_ptr(), Sa.data_ptr(), self.m_hat.data_ptr(), None, N, C, HW, float(self.eps),
          st)
        if residual is not None:
            from .resblock import triton_add_shortcut

            triton_add_shortcut(residual[0], residual[1], ma, Sa)
        return ma, Sa

    def backward(self, delta_ma: Tensor, delta_Sa: Tensor, relu=None,
                 delta_sums: bool = False) -> tuple[Tensor, Tensor]:
        """Input deltas and the γ/β sums; with ``relu`` (the ReLU layer that feeds
        this one in a container) the deltas leave already multiplied by its
        Jacobian, i.e. as ``relu.backward`` would return them. ``delta_sums``:
        the same launch also sums the outgoing deltas per channel (float64,
        means then variances) into ``self.delta_sums``: the bias sums of the
        convolution before, which a container hands to its backward."""
        check_cuda_f32(delta_ma, delta_Sa)
        dma, dSa = delta_ma.contiguous(), delta_Sa.contiguous()
        N, C, H, W = self.input_shape
        dev = dma.device
        st = stream(dma)
        L = lib()
        dmz = torch.empty_like(dma)
        dSz = torch.empty_like(dSa)
        mode = self._param_mode
        grads = (self._reducer.buffer(self, 4 * C, torch.float64) if mode == "sums"
                 else torch.empty(4 * C, device=dev, dtype=torch.float64))
        rj = None
        if relu is not None:
            if relu.J is None or relu.J.numel() != dma.numel():
                raise ValueError("BatchNorm2D.backward: the ReLU has no Jacobian of this size")
            rj = relu.J.contiguous()
        upd = mode == "update"  # the capped update applied by the same launch
        self.delta_sums = (torch.empty(2 * C, device=dev, dtype=torch.float64) if delta_sums
                           else None)
        L("tagi_bn_backward", dma.data_ptr(), dSa.data_ptr(), self.m_hat.data_ptr(),
          self._norm_var.data_ptr(), self.mw.data_ptr(), dmz.data_ptr(), dSz.data_ptr(),
          rj.data_ptr() if rj is not None else None, grads.data_ptr(),
          self.delta_sums.data_ptr() if delta_sums else None, N, C, H * W,
          float(self.eps), self.Sw.data_ptr() if upd else None,
          self.mb.data_ptr() if upd else None, self.Sb.data_ptr() if upd else None,
          float(self._cap) if upd else 0.0, st)
        if mode == "deltas":
            self.delta_mw = torch.empty(C, device=dev)
            self.delta_Sw = torch.empty(C, device=dev)
            self.delta_mb = torch.empty(C, device=dev)
            self.delta_Sb = torch.empty(C, device=dev)
            L("tagi_bn_apply_grads", grads.data_ptr(), C, WGRAD_DELTAS, None, self.Sw.data_ptr(),
              None, self.Sb.data_ptr(), self.delta_mw.data_ptr(), self.delta_Sw.data_ptr(),
              self.delta_mb.data_ptr(), self.delta_Sb.data_ptr(), 1.0, st)
        elif mode == "update":
            self._updated_in_backward = True
        elif mode == "sums":
            self._reducer.ready(self)
        else:
            raise ValueError(f"unknown parameter mode {mode!r}")
        return dmz, dSz

    def _sums_numel(self) -> int:
        return 4 * self.num_features

    def _apply_sums(self, grads: Tensor, cap: float) -> None:
        lib()("tagi_bn_apply_grads", grads.data_ptr(), self.num_features, WGRAD_UPDATE,
              self.mw.data_ptr(), self.Sw.data_ptr(), self.mb.data_ptr(), self.Sb.data_ptr(),
              None, None, None, None, float(cap), stream(grads))

    def update(self, cap_factor: float) -> None:
        from ..update.parameters import update_parameters

        if self._updated_in_backward:
            self._updated_in_backward = False
            return
        if self._param_mode == "sums":
            return
        update_parameters(self.mw, self.Sw, self.delta_mw, self.delta_Sw, cap_factor)
        update_parameters(self.mb, self.Sb, self.delta_mb, self.delta_Sb, cap_factor)

    @property
    def num_parameters(self) -> int:
        return 2 * (self.mw.numel() + self.mb.numel())

    def __repr__(self):
        return (f"BatchNorm2D(num_features={self.num_features}, momentum={self.momentum}, "
                f"eps={self.eps})")
