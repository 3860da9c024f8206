"""Parameter initialisation (drop-in for triton_tagi/param_init.py).

Same scales and draw order as the reference (which mirrors cuTAGI):
He scale √(1/fan_in), Xavier √(2/(fan_in+fan_out)); means ~ N(0, scale),
variances (gain·scale)²; norm layers γ = 1, β = 0 with variance 2/(2n)·gain².
Draws use torch's global RNG on the target device, as the reference does.
"""

from __future__ import annotations

import math

import torch


def he_init(fan_in: float) -> float:
    return math.sqrt(1.0 / fan_in)


def xavier_init(fan_in: float, fan_out: float) -> float:
    return math.sqrt(2.0 / (fan_in + fan_out))


def gaussian_param_init(scale: float, gain: float, shape, device="cuda"):
    m = torch.randn(shape, device=device) * scale
    S = torch.full(shape if isinstance(shape, tuple) else (shape,), (gain * scale) ** 2,
                   device=device)
    return m, S


def _scale(init_method: str, fan_in: float, fan_out: float) -> float:
    name = init_method.lower()
    if name == "xavier":
        return xavier_init(fan_in, fan_out)
    if name == "he":
        return he_init(fan_in)
    raise ValueError(f"Unsupported init method: {init_method}")


def init_weight_bias_linear(input_size, output_size, init_method="He", gain_w=1.0, gain_b=1.0,
                            bias=True, device="cuda"):
    scale = _scale(init_method, input_size, output_size)
    mw, Sw = gaussian_param_init(scale, gain_w, (input_size, output_size), device)
    if bias:
        mb, Sb = gaussian_param_init(scale, gain_b, (1, output_size), device)
    else:
        mb = torch.zeros(1, output_size, device=device)
        Sb = torch.zeros(1, output_size, device=device)
    return mw, Sw, mb, Sb


def init_weight_bias_conv2d(kernel_size, in_channels, out_channels, init_method="He", gain_w=1.0,
                            gain_b=1.0, device="cuda"):
    fan_in = kernel_size**2 * in_channels
    fan_out = kernel_size**2 * out_channels
    scale = _scale(init_method, fan_in, fan_out)
    K = in_channels * kernel_size * kernel_size
    mw, Sw = gaussian_param_init(scale, gain_w, (K, out_channels), device)
    mb, Sb = gaussian_param_init(scale, gain_b, (1, out_channels), device)
    return mw, Sw, mb, Sb


def init_weight_bias_norm(num_features, gain_w=1.0, gain_b=1.0, device="cuda"):
    scale = 2.0 / (num_features + num_features)
    return (torch.ones(num_features, device=device),
            torch.full((num_features,), scale * gain_w**2, device=device),
            torch.zeros(num_features, device=device),
            torch.full((num_features,), scale * gain_b**2, device=device))
