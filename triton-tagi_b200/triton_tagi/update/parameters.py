"""Capped closed-form parameter update (drop-in for triton_tagi/update/parameters.py).

    δ̄ = √max(S, 1e-10) / cap
    m ← m + sign(Δm)·min(|Δm|, δ̄)
    S ← S + sign(ΔS)·min(|ΔS|, δ̄), floored to 1e-5 when the result is ≤ 0
"""

from __future__ import annotations

from torch import Tensor

from .._lib import check_cuda_f32, lib, stream


def get_cap_factor(batch_size: int) -> float:
    """0.1 for batch 1, 2.0 below 256, 3.0 otherwise (parameters.py:30-50)."""
    if batch_size == 1:
        return 0.1
    return 2.0 if batch_size < 256 else 3.0


def update_parameters(m: Tensor, S: Tensor, delta_m: Tensor, delta_S: Tensor,
                      cap_factor: float) -> None:
    """In-place capped update of (m, S); all four tensors hold m.numel() floats
    and must be contiguous (the reference flattens them with ``.view(-1)``)."""
    check_cuda_f32(m, S, delta_m, delta_S)
    n = m.numel()
    for t in (S, delta_m, delta_S):
        if t.numel() != n:
            raise ValueError("update_parameters: size mismatch")
    mv, Sv = m.view(-1), S.view(-1)
    dm, dS = delta_m.reshape(-1).contiguous(), delta_S.reshape(-1).contiguous()
    lib()("tagi_capped_update", mv.data_ptr(), Sv.data_ptr(), dm.data_ptr(), dS.data_ptr(), n,
          float(cap_factor), stream(m))
