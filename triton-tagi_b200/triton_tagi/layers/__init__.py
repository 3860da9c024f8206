"""TAGI layers (drop-in for triton_tagi/layers)."""

from .avgpool2d import AvgPool2D
from .batchnorm2d import BatchNorm2D
from .conv2d import Conv2D
from .embedding import Embedding
from .flatten import Flatten
from .linear import Linear
from .multihead_attention import MultiheadAttentionV2
from .positional_encoding import PositionalEncoding
from .relu import ReLU
from .remax import Remax
from .resblock import Add, ResBlock
from .rms_norm import RMSNorm

__all__ = ["Add", "AvgPool2D", "BatchNorm2D", "Conv2D", "Embedding", "Flatten", "Linear",
           "MultiheadAttentionV2", "PositionalEncoding", "RMSNorm", "ReLU", "Remax", "ResBlock"]
