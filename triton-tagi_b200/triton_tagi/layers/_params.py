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
                          transposed: bool = False, bias_sums=None) -> None:
    """Parameter side of backward for a (K x N) weight and optional (1 x N) bias.

    a: activation matrix (M x K, row stride lda), or with ``transposed`` its
    transpose (K x M, row stride lda); dm = (dmz, dSz) with row map
    d_map = (div, outer, stride, col_stride). ``bias_sums``: the bias's two
    column sums of (dmz, dSz), already computed (float64, 2 N values); the
    contraction then covers the weight rows only.
    """
    contiguous_params(layer)
    dmz, dSz = dm
    mode = layer._param_mode
    L = lib()
    hb = 1 if has_bias else 0
    if bias_sums is not None and (not has_bias or bias_sums.numel() != 2 * N
                                  or bias_sums.dtype != torch.float64):
        raise ValueError("bias_sums must hold 2 * N float64 values of a layer with a bias")
    hold, wp, wn = workspace(L.size("tagi_param_grad_workspace_size", M, K, N, hb), a)
    head = (dmz.data_ptr(), dSz.data_ptr(), *d_map, M, K, N)

    def run(code, params, outs, cap):
        if bias_sums is None:
            L("tagi_param_grad_t" if transposed else "tagi_param_grad", a.data_ptr(), lda, *head,
              hb, code, *params, *outs, cap, wp, wn, stream(a))
        else:
            L("tagi_param_grad_bias_given", a.data_ptr(), lda, 1 if transposed else 0, *head,
              bias_sums.data_ptr(), code, *params, *outs, cap, wp, wn, stream(a))

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
        run(WGRAD_DELTAS, (None, layer.Sw.data_ptr(), None,
                           layer.Sb.data_ptr() if has_bias else None), outs, 1.0)
    elif mode == "update":
        run(WGRAD_UPDATE, (layer.mw.data_ptr(), layer.Sw.data_ptr(),
                           layer.mb.data_ptr() if has_bias else None,
                           layer.Sb.data_ptr() if has_bias else None), null4, float(layer._cap))
        layer._updated_in_backward = True
    elif mode == "sums":
        buf = layer._reducer.buffer(layer, sums_numel(K, N, has_bias), torch.float32)
        half = buf.numel() // 2
        run(WGRAD_SUMS, null4, (buf.data_ptr(), buf[half:].data_ptr(), None, None), 1.0)
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
