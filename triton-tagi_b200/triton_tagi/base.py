"""Layer contract (drop-in for triton_tagi/base.py:21-67).

``Layer`` propagates Gaussian moments forward and innovation deltas backward;
``LearnableLayer`` adds ``update(cap_factor)`` and ``num_parameters``.

Learnable layers also carry a *parameter mode* that decides what ``backward``
does with the batch sums aᵀ·δ it computes:

* ``"deltas"`` (default, the reference behaviour): store ``delta_mw``,
  ``delta_Sw``, ``delta_mb``, ``delta_Sb``; ``update(cap)`` applies them.
* ``"update"``: apply the capped update inside ``backward`` (after the
  deltas for the previous layer have been propagated with the pre-update
  weights), so the weight-gradient kernel writes parameters directly and no
  delta tensors are materialised. ``Sequential.step`` uses this on one GPU;
  the result equals backward-then-update because each layer's update touches
  only its own parameters.
* ``"sums"``: write the raw batch sums into buffers owned by a data-parallel
  reducer; the update is applied after the sums were all-reduced.
"""

from __future__ import annotations

from abc import ABC, abstractmethod

from torch import Tensor


class Layer(ABC):
    """Base class for all TAGI layers."""

    @abstractmethod
    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        """Propagate activation means and variances forward."""

    @abstractmethod
    def backward(self, delta_ma: Tensor, delta_Sa: Tensor) -> tuple[Tensor, Tensor]:
        """Propagate innovation deltas backward; returns deltas for the previous layer."""


class LearnableLayer(Layer):
    """Base class for layers with trainable Gaussian parameters."""

    _param_mode: str = "deltas"
    _cap: float | None = None
    _reducer = None
    # Set by Sequential.step on its first layer while it runs backward: the input
    # deltas that backward returns are discarded there, so layers that honour it
    # skip computing them (and return None) but still form their parameter sums.
    _skip_input_delta: bool = False
    _updated_in_backward: bool = False

    @abstractmethod
    def update(self, cap_factor: float) -> None:
        """Apply the capped parameter update using what backward stored."""

    @property
    @abstractmethod
    def num_parameters(self) -> int:
        """Number of learnable scalars (means and variances)."""

    # -- parameter-mode plumbing (used by Sequential) ---------------------------
    def _leaves(self) -> list["LearnableLayer"]:
        """Learnable layers that own parameters directly (composites override)."""
        return [self]

    def _set_param_mode(self, mode: str, cap: float | None = None, reducer=None) -> None:
        for leaf in self._leaves():
            leaf._param_mode, leaf._cap, leaf._reducer = mode, cap, reducer
            leaf._updated_in_backward = False
