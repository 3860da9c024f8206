"""Batched TAGI products for MultiheadAttentionV2.

Drop-in for triton_tagi/kernels/attention.py (bmm_tagi_var 149-201,
bmm_shared_right 286-336, bmm_shared_left 339-374): same signatures, same
stride rules (leading dims packed; ``transpose(-1, -2)`` views accepted
without copies), computed by libtagi_b200. ``bmm_shared_left`` returns
contiguous tensors where the reference returns transposed views of them.
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream


def _batch_stride(x: Tensor) -> int:
    """Stride between flattened leading-dim slices (leading dims must be packed)."""
    return x.numel() if x.dim() <= 2 else x.stride(-3)


def _nbatch(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def _packed(x: Tensor) -> Tensor:
    """Leading dims must advance by stride(-3); otherwise make a contiguous copy."""
    if x.dim() <= 3:
        return x
    expect = x.stride(-3)
    for d in range(x.dim() - 4, -1, -1):
        expect *= x.shape[d + 1]
        if x.stride(d) != expect and x.shape[d] != 1:
            return x.contiguous()
    return x


def bmm_tagi_var(mu_a: Tensor, var_a: Tensor, mu_b: Tensor, var_b: Tensor,
                 scale_sq: float = 1.0) -> Tensor:
    """var[..., m, l] = scale_sq · Σ_k var_a (μ_b² + var_b) + μ_a² var_b."""
    return bmm_tagi_moments(mu_a, var_a, mu_b, var_b, None, scale_sq)[1]


def bmm_tagi_moments(mu_a: Tensor, var_a: Tensor, mu_b: Tensor, var_b: Tensor,
                     scale: float | None, scale_sq: float) -> tuple[Tensor | None, Tensor]:
    """Variance as in ``bmm_tagi_var`` and, when ``scale`` is given, the mean
    scale · μ_a @ μ_b from the same pass (replaces the separate mean matmul of
    triton_tagi/layers/multihead_attention.py:180, 192)."""
    check_cuda_f32(mu_a, var_a, mu_b, var_b)
    batch_shape = mu_a.shape[:-2]
    M, K = mu_a.shape[-2:]
    Kb, L = mu_b.shape[-2:]
    if K != Kb:
        raise ValueError(f"Reduction dims disagree: a has {K}, b has {Kb}")
    mu_a, var_a, mu_b, var_b = (_packed(t) for t in (mu_a, var_a, mu_b, var_b))
    if var_a.stride() != mu_a.stride():
        mu_a, var_a = mu_a.contiguous(), var_a.contiguous()
    if var_b.stride() != mu_b.stride():
        mu_b, var_b = mu_b.contiguous(), var_b.contiguous()
    N = _nbatch(batch_shape)
    var = torch.empty((*batch_shape, M, L), device=mu_a.device, dtype=mu_a.dtype)
    mean = torch.empty_like(var) if scale is not None else None
    lib()("tagi_bmm_tagi_var", mu_a.data_ptr(), var_a.data_ptr(), mu_b.data_ptr(),
          var_b.data_ptr(), None if mean is None else mean.data_ptr(), var.data_ptr(), N, M, L, K,
          _batch_stride(mu_a), mu_a.stride(-2), mu_a.stride(-1), _batch_stride(mu_b),
          mu_b.stride(-2), mu_b.stride(-1), _batch_stride(var), var.stride(-2), var.stride(-1),
          1.0 if scale is None else scale, scale_sq, stream(mu_a))
    return mean, var


def bmm_shared_right(a_mean: Tensor, a_var: Tensor, b: Tensor,
                     scale: float = 1.0) -> tuple[Tensor, Tensor]:
    """mean = scale · a_mean @ b, var = scale² · a_var @ b² (b deterministic)."""
    check_cuda_f32(a_mean, a_var, b)
    batch_shape = a_mean.shape[:-2]
    M, K = a_mean.shape[-2:]
    Kb, L = b.shape[-2:]
    if K != Kb:
        raise ValueError(f"Reduction dims disagree: a has {K}, b has {Kb}")
    a_mean, a_var, b = (_packed(t) for t in (a_mean, a_var, b))
    if a_var.stride() != a_mean.stride():
        a_mean, a_var = a_mean.contiguous(), a_var.contiguous()
    N = _nbatch(batch_shape)
    mean = torch.empty((*batch_shape, M, L), device=a_mean.device, dtype=a_mean.dtype)
    var = torch.empty_like(mean)
    lib()("tagi_bmm_shared_right", a_mean.data_ptr(), a_var.data_ptr(), b.data_ptr(),
          mean.data_ptr(), var.data_ptr(), N, M, L, K, _batch_stride(a_mean), a_mean.stride(-2),
          a_mean.stride(-1), _batch_stride(b), b.stride(-2), b.stride(-1), _batch_stride(mean),
          mean.stride(-2), mean.stride(-1), scale, stream(a_mean))
    return mean, var


def bmm_shared_left(a: Tensor, b_mean: Tensor, b_var: Tensor,
                    scale: float = 1.0) -> tuple[Tensor, Tensor]:
    """mean = scale · a @ b_mean, var = scale² · a² @ b_var (a deterministic).

    The reference evaluates this through its shared-right kernel on
    (b_meanᵀ, b_varᵀ, aᵀ) (attention.py:364-374); here one contraction squares
    the left operand (tagi_bmm_shared_left), so the output rows are a's rows
    (the S score rows of the attention value deltas, not the head dimension)
    and the result comes back contiguous, not as a transposed view.
    """
    check_cuda_f32(a, b_mean, b_var)
    batch_shape = a.shape[:-2]
    M, K = a.shape[-2:]
    Kb, L = b_mean.shape[-2:]
    if K != Kb:
        raise ValueError(f"Reduction dims disagree: a has {K}, b has {Kb}")
    a, b_mean, b_var = (_packed(t) for t in (a, b_mean, b_var))
    if b_var.stride() != b_mean.stride():
        b_mean, b_var = b_mean.contiguous(), b_var.contiguous()
    N = _nbatch(batch_shape)
    mean = torch.empty((*batch_shape, M, L), device=a.device, dtype=a.dtype)
    var = torch.empty_like(mean)
    lib()("tagi_bmm_shared_left", a.data_ptr(), b_mean.data_ptr(), b_var.data_ptr(),
          mean.data_ptr(), var.data_ptr(), N, M, L, K, _batch_stride(a), a.stride(-2),
          a.stride(-1), _batch_stride(b_mean), b_mean.stride(-2), b_mean.stride(-1),
          _batch_stride(mean), mean.stride(-2), mean.stride(-1), scale, stream(a))
    return mean, var
