"""Moment-contraction kernels (sm_100a CUDA through the C ABI).

Function names and signatures follow triton_tagi/kernels/__init__.py of the
reference so existing callers work unchanged; there is no Triton underneath.
"""

from .attention import bmm_shared_left, bmm_shared_right, bmm_tagi_var
from .common import triton_fused_backward_delta, triton_fused_var_forward, triton_fused_weight_grad

__all__ = [
    "bmm_shared_left",
    "bmm_shared_right",
    "bmm_tagi_var",
    "triton_fused_backward_delta",
    "triton_fused_var_forward",
    "triton_fused_weight_grad",
]
