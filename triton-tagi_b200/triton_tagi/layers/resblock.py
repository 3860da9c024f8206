"""Residual block and Add (drop-in for triton_tagi/layers/resblock.py).

Main path Conv(3×3, stride) → ReLU → BN → Conv(3×3) → ReLU → BN; shortcut is
the identity or, when stride > 1 or channels change, Conv(2×2, stride) → ReLU
→ BN; the two are added (means and variances) with no activation after
(resblock.py:354-385). Backward sends the incoming deltas down both branches
and sums what comes back (resblock.py:390-430). Stride-2 blocks use
right/bottom padding on their first convolution (resblock.py:272-282).
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream
from ..base import LearnableLayer
from .batchnorm2d import BatchNorm2D
from .conv2d import Conv2D
from .relu import ReLU


def triton_add_shortcut(mu_s: Tensor, var_s: Tensor, mu_a: Tensor, var_a: Tensor) -> None:
    """In place: mu_a += mu_s, var_a += var_s (resblock.py:138-154)."""
    if mu_s.shape != mu_a.shape:
        raise ValueError(f"Shape mismatch: shortcut={tuple(mu_s.shape)} vs output={tuple(mu_a.shape)}")
    check_cuda_f32(mu_s, var_s, mu_a, var_a)
    if not (mu_a.is_contiguous() and var_a.is_contiguous()):
        raise ValueError("in-place targets must be contiguous")
    mu_s, var_s = mu_s.contiguous(), var_s.contiguous()
    lib()("tagi_add_inplace", mu_a.data_ptr(), var_a.data_ptr(), mu_s.data_ptr(),
          var_s.data_ptr(), mu_a.numel(), stream(mu_a))


triton_delta_merge = triton_add_shortcut  # resblock.py:157-175 (same arithmetic)


class Add:
    """Element-wise sum of two Gaussian streams (resblock.py:183-213)."""

    def forward(self, mu_z, var_z, mu_x, var_x):
        if mu_z.shape != mu_x.shape:
            raise ValueError("Add: shape mismatch")
        mu_s, var_s = mu_z.clone(), var_z.clone()
        triton_add_shortcut(mu_x, var_x, mu_s, var_s)
        return mu_s, var_s

    def backward(self, delta_mu_s, delta_var_s):
        return ((delta_mu_s.clone(), delta_var_s.clone()),
                (delta_mu_s.clone(), delta_var_s.clone()))

    def __repr__(self):
        return "Add()"


class ResBlock(LearnableLayer):
    def __init__(self, in_channels: int, out_channels: int, stride: int = 1, device="cuda",
                 gain_w: float = 1.0, gain_b: float = 1.0) -> None:
        self.in_channels, self.out_channels, self.stride = in_channels, out_channels, stride
        self.device = device
        self.training = True
        kw = dict(device=device, gain_w=gain_w, gain_b=gain_b)
        self.conv1 = Conv2D(in_channels, out_channels, kernel_size=3, stride=stride, padding=1,
                            padding_type=2 if stride > 1 else 1, **kw)
        self.relu1 = ReLU()
        self.bn1 = BatchNorm2D(out_channels, preserve_var=False, **kw)
        self.conv2 = Conv2D(out_channels, out_channels, kernel_size=3, stride=1, padding=1, **kw)
        self.relu2 = ReLU()
        self.bn2 = BatchNorm2D(out_channels, preserve_var=False, **kw)
        self._main_layers = [self.conv1, self.relu1, self.bn1, self.conv2, self.relu2, self.bn2]
        self.use_projection = (stride != 1) or (in_channels != out_channels)
        if self.use_projection:
            self.proj_conv = Conv2D(in_channels, out_channels, kernel_size=2, stride=stride,
                                    padding=0, **kw)
            self.proj_relu = ReLU()
            self.proj_bn = BatchNorm2D(out_channels, preserve_var=False, **kw)
            self._proj_layers = [self.proj_conv, self.proj_relu, self.proj_bn]
        else:
            self.proj_conv = self.proj_relu = self.proj_bn = None
            self._proj_layers = []
        self._learnable = [self.conv1, self.bn1, self.conv2, self.bn2]
        if self.use_projection:
            self._learnable += [self.proj_conv, self.proj_bn]

    def _leaves(self):
        return list(self._learnable)

    def train(self) -> None:
        self.training = True
        for layer in self._learnable:
            if hasattr(layer, "train"):
                layer.train()

    def eval(self) -> None:
        self.training = False
        for layer in self._learnable:
            if hasattr(layer, "eval"):
                layer.eval()

    def forward(self, mu_in: Tensor, var_in: Tensor) -> tuple[Tensor, Tensor]:
        # Layers never modify their inputs, so the skip needs no copy.
        from .._chain import forward_chain

        # shortcut first: the main path's last BatchNorm adds it to its outputs
        mu_x, var_x = forward_chain(self._proj_layers, mu_in, var_in)
        mu_z, var_z = forward_chain(self._main_layers[:-1], mu_in, var_in)
        return self._main_layers[-1].forward(mu_z, var_z, residual=(mu_x, var_x))

    def backward(self, delta_mu: Tensor, delta_var: Tensor) -> tuple[Tensor, Tensor]:
        from .._chain import backward_chain

        d_mu_main, d_var_main = backward_chain(self._main_layers, delta_mu, delta_var)
        d_mu_skip, d_var_skip = backward_chain(self._proj_layers, delta_mu, delta_var)
        triton_delta_merge(d_mu_skip, d_var_skip, d_mu_main, d_var_main)
        return d_mu_main, d_var_main

    def update(self, cap_factor: float) -> None:
        for layer in self._learnable:
            layer.update(cap_factor)

    @property
    def mw(self):
        return self.conv1.mw

    @mw.setter
    def mw(self, value):
        self.conv1.mw = value

    @property
    def Sw(self):
        return self.conv1.Sw

    @property
    def mb(self):
        return self.conv1.mb

    @property
    def Sb(self):
        return self.conv1.Sb

    @property
    def num_parameters(self) -> int:
        return sum(layer.num_parameters for layer in self._learnable)

    def __repr__(self):
        proj = "projection" if self.use_projection else "identity"
        return f"ResBlock({self.in_channels}→{self.out_channels}, stride={self.stride}, skip={proj})"
