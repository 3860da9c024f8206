"""Flatten (N, C, H, W) ↔ (N, C·H·W) (drop-in for triton_tagi/layers/flatten.py)."""

from __future__ import annotations

from torch import Tensor

from ..base import Layer


class Flatten(Layer):
    def __init__(self) -> None:
        self.shape = None

    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        self.shape = ma.shape
        N = ma.shape[0]
        return ma.reshape(N, -1), Sa.reshape(N, -1)

    def backward(self, delta_m: Tensor, delta_S: Tensor) -> tuple[Tensor, Tensor]:
        return delta_m.reshape(self.shape), delta_S.reshape(self.shape)

    def __repr__(self):
        return "Flatten()"
