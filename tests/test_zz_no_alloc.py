"""The weight-sum entry point that allocates nothing (tagi_fused_weight_grad_static).

Some callers cannot give the library scratch memory: a host runtime that binds
this library through a plain C FFI has no CUDA allocator of its own, and an
application running from a fixed device-memory pool may forbid a plugin to
grow it. For them the split-reduction weight sums keep their partials in an
array inside the library's device image instead of a caller workspace. These
tests call that entry point through the C ABI, twice in a row with different
split plans, and compare it with the workspace entry point; a shape whose plan
needs more than the array must be refused with an error.

This file is named so that pytest collects it last.
"""

from __future__ import annotations

import re

import pytest
import torch

from _tol import MEAN_RTOL, VAR_RTOL, assert_rel

pytestmark = pytest.mark.gpu
DEV = "cuda"
STATIC_BYTES = 16 << 20


def _static_call(a, dmz, dSz):
    from triton_tagi._lib import lib, stream

    M, K = a.shape
    N = dmz.shape[1]
    gm = torch.empty(K, N, device=a.device)
    gS = torch.empty(K, N, device=a.device)
    lib()("tagi_fused_weight_grad_static", a.data_ptr(), dmz.data_ptr(), dSz.data_ptr(),
          gm.data_ptr(), gS.data_ptr(), M, K, N, a.stride(0), a.stride(1), dmz.stride(0),
          dmz.stride(1), gm.stride(0), gm.stride(1), stream(a))
    return gm, gS


def _inputs(M, K, N, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g)
    dmz = torch.randn(M, N, generator=g) * 0.1
    dSz = -torch.rand(M, N, generator=g) * 1e-2
    return a.to(DEV), dmz.to(DEV), dSz.to(DEV)


def test_static_scratch_matches_workspace_entry_point_on_consecutive_calls():
    from triton_tagi._lib import lib
    from triton_tagi.kernels.common import triton_fused_weight_grad

    L = lib()
    # two calls in a row with different split plans (the first on the tensor-core
    # kernel, the second on CUDA cores); the second reuses the array
    for seed, (M, K, N) in enumerate([(131072, 288, 32), (50000, 27, 10)]):
        # both entry points hold the split partials and, where room is left after
        # them, the tensor-core kernel's prepared delta tiles in their scratch
        assert L.size("tagi_fused_weight_grad_workspace_size", M, K, N) > 0
        a, dmz, dSz = _inputs(M, K, N, seed)
        ref_m, ref_S = triton_fused_weight_grad(a, dmz, dSz)
        got_m, got_S = _static_call(a, dmz, dSz)
        torch.cuda.synchronize()
        assert_rel(got_m, ref_m, MEAN_RTOL, f"call {seed}: grad_mw")
        assert_rel(got_S, ref_S, VAR_RTOL, f"call {seed}: grad_Sw")


def test_static_scratch_refuses_shapes_beyond_its_size():
    from triton_tagi._lib import lib

    L = lib()
    M, K, N = 8192, 2304, 512  # two-way split plan: 18.9 MB of partial sums
    # the size query reports partials plus prepared tiles; the refusal is decided
    # on the partials alone, whose size the error message states
    assert L.size("tagi_fused_weight_grad_workspace_size", M, K, N) > STATIC_BYTES
    a, dmz, dSz = _inputs(M, K, N, 7)
    with pytest.raises(RuntimeError, match="static") as err:
        _static_call(a, dmz, dSz)
    need = int(re.search(r"needs (\d+) bytes", str(err.value)).group(1))
    assert need > STATIC_BYTES, need
