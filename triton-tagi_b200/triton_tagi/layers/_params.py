"""Shared parameter-side backward for the weight layers (Linear, Conv2D).

One call of ``tagi_param_grad`` forms the batch sums aᵀ·δμ and (a²)ᵀ·δS
(with the bias as an extra row of ones) and, depending on the layer's
parameter mode, stores the reference's delta tensors
(triton_tagi/layers/linear.py:138-151), applies the capped update in place
(triton_tagi/update/parameters.py:77-96), or writes raw sums for an
all-reduce.
"""

from __future__ import annotations

import torch

from .._lib import WGRAD_DELTAS, WGRAD_SUMS, WGRAD_UPDATE, lib, stream, workspace


def contiguous_params(layer, names=("mw", "Sw", "mb", "Sb")) -> None:
    """Parameters are updated in place by the kernels, so keep them contiguous."""
    for n in names:
        t = getattr(layer, n, None)
        if t is not None and not t.is_contiguous():
            setattr(layer, n, t.contiguous())


def sums_numel(K: int, N: int, has_bias: bool) -> int:
    return 2 * (K + (1 if has_bias else 0)) * N


def weight_param_backward(layer, a, lda, dm, d_map, M, K, N, has_bias,
                          transposed: bool = False) -> None:
    """Parameter side of backward for a (K x N) weight and optional (1 x N) bias.

    a: activation matrix (M x K, row stride lda), or with ``transposed`` its
    transpose (K x M, row stride lda); dm = (dmz, dSz) with row map
    d_map = (div, outer, stride, col_stride).
    """
    contiguous_params(layer)
    dmz, dSz = dm
    mode = layer._param_mode
    L = lib()
    entry = "tagi_param_grad_t" if transposed else "tagi_param_grad"
    hb = 1 if has_bias else 0
    hold, wp, wn = workspace(L.size("tagi_param_grad_workspace_size", M, K, N, hb), a)
    null4 = (None, None, None, None)
    if mode == "deltas":
        dev = a.device
        layer.delta_mw = torch.empty(K, N, device=dev)
        layer.delta_Sw = torch.empty(K, N, device=dev)
        if has_bias:
            layer.delta_mb = torch.empty(1, N, device=dev)
            layer.delta_Sb = torch.empty(1, N, device=dev)
        outs = (layer.delta_mw.data_ptr(), layer.delta_Sw.data_ptr(),
                layer.delta_mb.data_ptr() if has_bias else None,
                layer.delta_Sb.data_ptr() if has_bias else None)
        L(entry, a.data_ptr(), lda, dmz.data_ptr(), dSz.data_ptr(), *d_map, M, K, N,
          hb, WGRAD_DELTAS, None, layer.Sw.data_ptr(), None,
          layer.Sb.data_ptr() if has_bias else None, *outs, 1.0, wp, wn, stream(a))
    elif mode == "update":
        L(entry, a.data_ptr(), lda, dmz.data_ptr(), dSz.data_ptr(), *d_map, M, K, N,
          hb, WGRAD_UPDATE, layer.mw.data_ptr(), layer.Sw.data_ptr(),
          layer.mb.data_ptr() if has_bias else None, layer.Sb.data_ptr() if has_bias else None,
          *null4, float(layer._cap), wp, wn, stream(a))
        layer._updated_in_backward = True
    elif mode == "sums":
        buf = layer._reducer.buffer(layer, sums_numel(K, N, has_bias), torch.float32)
        half = buf.numel() // 2
        L(entry, a.data_ptr(), lda, dmz.data_ptr(), dSz.data_ptr(), *d_map, M, K, N,
          hb, WGRAD_SUMS, None, None, None, None, buf.data_ptr(), buf[half:].data_ptr(), None,
          None, 1.0, wp, wn, stream(a))
        layer._reducer.ready(layer)
    else:
        raise ValueError(f"unknown parameter mode {mode!r}")
    del hold


def weight_apply_sums(layer, buf, K: int, N: int, has_bias: bool, cap: float) -> None:
    """Capped update from all-reduced sums (layout of ``weight_param_backward``)."""
    half = buf.numel() // 2
    lib()("tagi_apply_param_sums", buf.data_ptr(), buf[half:].data_ptr(), K, N,
          1 if has_bias else 0, layer.mw.data_ptr(), layer.Sw.data_ptr(),
          layer.mb.data_ptr() if has_bias else None, layer.Sb.data_ptr() if has_bias else None,
          float(cap), stream(buf))


def weight_update(layer, cap: float, has_bias: bool) -> None:
    """``update(cap)`` of the weight layers."""
    from ..update.parameters import update_parameters

    if layer._updated_in_backward:
        layer._updated_in_backward = False
        return
    if layer._param_mode == "sums":
        return  # applied by the data-parallel reducer after the all-reduce
    update_parameters(layer.mw, layer.Sw, layer.delta_mw, layer.delta_Sw, cap)
    if has_bias:
        update_parameters(layer.mb, layer.Sb, layer.delta_mb, layer.delta_Sb, cap)
