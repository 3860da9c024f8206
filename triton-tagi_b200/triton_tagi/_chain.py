"""Forward and backward passes over a chain of layers, with the fusions a
container may apply between neighbours (the results are the layers' own):

* a BatchNorm2D directly after a ReLU multiplies its outgoing deltas by the
  ReLU's Jacobian inside its backward, and the ReLU's own backward is skipped;
* a Conv2D whose outputs reach a BatchNorm2D (directly or through that ReLU)
  takes its bias sums (the per-channel sums of its output deltas) from the
  BatchNorm's backward launch instead of a pass of its own.

Forward fusions of the ReLU were measured and dropped: applied in the epilogue
of the contraction before it, the exp/erf of the rectified moments at the end of
every tile cost more than the memory-bound pass they replace; applied inside the
following BatchNorm's statistics and normalisation passes, it is evaluated
twice and made those passes slower by about as much as the ReLU pass costs.

Layers called one by one keep the reference's behaviour; only containers
(``Sequential``, ``ResBlock``) walk their layers through these functions.
"""

from __future__ import annotations

from torch import Tensor

from .base import Layer
from .layers.batchnorm2d import BatchNorm2D
from .layers.conv2d import Conv2D
from .layers.relu import ReLU


def forward_chain(layers, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
    for layer in layers:
        if not isinstance(layer, Layer):
            raise TypeError(f"Unknown layer type: {type(layer)}")
        ma, Sa = layer.forward(ma, Sa)
    return ma, Sa


def _conv_before(layers, i):
    """The Conv2D at layers[i] if it has a bias and computes parameter sums."""
    if i < 0:
        return None
    layer = layers[i]
    return layer if isinstance(layer, Conv2D) and layer.has_bias else None


def backward_chain(layers, dm: Tensor, dS: Tensor) -> tuple[Tensor, Tensor]:
    i = len(layers) - 1
    bias_sums = None  # for layers[i], from the BatchNorm after it
    while i >= 0:
        layer = layers[i]
        prev = layers[i - 1] if i > 0 else None
        if (isinstance(layer, BatchNorm2D) and isinstance(prev, ReLU) and prev.J is not None
                and prev.J.numel() == dm.numel()):
            conv = _conv_before(layers, i - 2)
            dm, dS = layer.backward(dm, dS, relu=prev, delta_sums=conv is not None)
            bias_sums = layer.delta_sums
            i -= 2
        elif isinstance(layer, BatchNorm2D):
            conv = _conv_before(layers, i - 1)
            dm, dS = layer.backward(dm, dS, delta_sums=conv is not None)
            bias_sums = layer.delta_sums
            i -= 1
        elif bias_sums is not None and isinstance(layer, Conv2D):
            dm, dS = layer.backward(dm, dS, bias_sums=bias_sums)
            bias_sums = None
            i -= 1
        else:
            dm, dS = layer.backward(dm, dS)
            bias_sums = None
            i -= 1
    return dm, dS
