"""triton-tagi API on a B200-native implementation.

Tractable Approximate Gaussian Inference with every moment kernel implemented
as hand-written sm_100a CUDA (libtagi_b200.so, reached through a C ABI). The
module layout and public names follow the reference package so that existing
code switches by changing nothing but the installation. There is no Triton and
no CPU path: tensors must be float32 on a CUDA device.
"""

from .base import Layer, LearnableLayer
from .layers import (Add, AvgPool2D, BatchNorm2D, Conv2D, Embedding, Flatten, Linear,
                     MultiheadAttentionV2, PositionalEncoding, ReLU, Remax, ResBlock, RMSNorm)
from .network import Sequential
from .checkpoint import RunDir, load_model
from .param_init import (gaussian_param_init, he_init, init_weight_bias_conv2d,
                         init_weight_bias_linear, init_weight_bias_norm, xavier_init)

__version__ = "0.1.0"
__all__ = [
    "Layer", "LearnableLayer", "Sequential", "RunDir", "load_model",
    "Add", "AvgPool2D", "BatchNorm2D", "Conv2D", "Embedding", "Flatten", "Linear",
    "MultiheadAttentionV2", "PositionalEncoding", "RMSNorm", "ReLU", "Remax", "ResBlock",
    "he_init", "xavier_init", "gaussian_param_init", "init_weight_bias_linear",
    "init_weight_bias_conv2d", "init_weight_bias_norm",
]
