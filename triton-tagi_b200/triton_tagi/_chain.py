"""Forward and backward passes over a chain of layers, with the fusions a
container may apply between neighbours (the results are the layers' own):

* a BatchNorm2D directly after a ReLU multiplies its outgoing deltas by the
  ReLU's Jacobian inside its backward, and the ReLU's own backward is skipped.

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
from .layers.relu import ReLU


def forward_chain(layers, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
    for layer in layers:
        if not isinstance(layer, Layer):
            raise TypeError(f"Unknown layer type: {type(layer)}")
        ma, Sa = layer.forward(ma, Sa)
    return ma, Sa


def backward_chain(layers, dm: Tensor, dS: Tensor) -> tuple[Tensor, Tensor]:
    i = len(layers) - 1
    while i >= 0:
        layer = layers[i]
        prev = layers[i - 1] if i > 0 else None
        if (isinstance(layer, BatchNorm2D) and isinstance(prev, ReLU) and prev.J is not None
                and prev.J.numel() == dm.numel()):
            dm, dS = layer.backward(dm, dS, relu=prev)
            i -= 2
        else:
            dm, dS = layer.backward(dm, dS)
            i -= 1
    return dm, dS
