"""TAGI update rules: observation innovation and parameter updates."""

from .observation import compute_innovation
from .parameters import get_cap_factor, update_parameters

__all__ = ["compute_innovation", "get_cap_factor", "update_parameters"]
