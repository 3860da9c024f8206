"""The tensor-core kernels' abort path, taken on purpose.

Every wait inside the tcgen05 contraction kernel is bounded; when one runs out
the kernel records the error word read by ``tagi_device_status``, tells the
other CTA of its pair, stops issuing work, waits for its own MMAs and copies in
flight and frees its tensor memory before returning. The test hook
``tagi_set_wait_limit_ns`` with a value below one microsecond makes every
launch take that path from its start (the MMA issuer gives up before its first
stage; the producers and accumulator warps find the abort flag when their next
wait does not complete). The test checks that the call returns, that the error
word reports it, and that after restoring the default limit the same
contraction is correct again. No fault is involved: nothing waits on a barrier
that cannot complete except through the bounded, abort-aware waits.
"""

from __future__ import annotations

import pytest
import torch

import oracle.moments as F
from _tol import MEAN_RTOL, VAR_RTOL, assert_rel

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_wait_limit_runs_out_then_recovers():
    from triton_tagi import Linear
    from triton_tagi._lib import device_status, set_wait_limit_ns

    M, K, N = 4096, 1024, 1024  # routes to the tensor-core kernel (prepared weight tiles)
    g = torch.Generator().manual_seed(5)
    ma, Sa = torch.randn(M, K, generator=g), torch.rand(M, K, generator=g) * 1e-2 + 1e-4
    mw, Sw = torch.randn(K, N, generator=g) / K**0.5, torch.rand(K, N, generator=g) / K
    mb, Sb = torch.zeros(1, N), torch.full((1, N), 1e-3)
    lin = Linear(K, N, device=DEV)
    lin.mw, lin.Sw, lin.mb, lin.Sb = (t.to(DEV) for t in (mw, Sw, mb, Sb))
    a, s = ma.to(DEV), Sa.to(DEV)
    assert device_status(reset=True) == 0
    set_wait_limit_ns(1)
    try:
        lin.forward(a, s)
        torch.cuda.synchronize()
        code = device_status(reset=True)
    finally:
        set_wait_limit_ns(0)
    assert code != 0, "the forced abort was not reported"
    for _ in range(2):
        mz, Sz = lin.forward(a, s)
        torch.cuda.synchronize()
        assert device_status(reset=True) == 0
        d = lambda t: t.double()  # noqa: E731
        assert_rel(mz, F.mean_forward(d(ma), d(mw), d(mb)), MEAN_RTOL, "mz after recovery")
        assert_rel(Sz, F.var_forward(d(ma), d(Sa), d(mw), d(Sw), d(Sb)), VAR_RTOL,
                   "Sz after recovery")
