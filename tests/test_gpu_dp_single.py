"""The data-parallel step on one GPU: a one-rank NCCL process group.

With a single rank the all-reduces are identities, so a ``DataParallel``
network must reproduce the plain single-GPU step: the parameter sums written
for the reducer (bucketed after the first step) and applied after the
backward, and BatchNorm's SyncBN path (channel sums, all-reduce,
``tagi_bn_sync_forward``, the sums exchanged through the NVLink peer-memory
kernel, here with one rank) instead of the one-launch cluster forward. The same
is checked with the data-parallel step captured in a CUDA graph
(``capturable=True``), NCCL calls included. The graph is released before the
process group is destroyed.
"""

from __future__ import annotations

import datetime
import os
import tempfile

import pytest
import torch
import torch.distributed as dist

import oracle.net as ON  # noqa: F401  (keeps the import order of the other GPU tests)
import triton_tagi as TT
from _nets import build_config, copy_params, params
from _tol import rel_err, var_update_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def one_rank_group():
    fd, path = tempfile.mkstemp(prefix="tagi_nccl_")
    os.close(fd)
    os.unlink(path)
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", init_method=f"file://{path}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60))
    yield
    dist.destroy_process_group()


@pytest.mark.parametrize("graph", [False, True])
def test_one_rank_data_parallel_equals_plain_step(one_rank_group, graph):
    from triton_tagi.distributed import DataParallel

    torch.manual_seed(3)
    plain = build_config("r18", TT, device=DEV, width=0.25)
    dp_layers = build_config("r18", TT, device=DEV, width=0.25)
    copy_params(plain, dp_layers, DEV)
    net_p = TT.Sequential(plain, device=DEV)
    net_d = TT.Sequential(dp_layers, device=DEV, cuda_graph=graph)
    dp = DataParallel(net_d, capturable=graph, bucket_bytes=64 << 10)
    gen = torch.Generator().manual_seed(9)
    try:
        for step in range(4):
            x = torch.randn(16, 3, 32, 32, generator=gen).to(DEV)
            y = torch.nn.functional.one_hot(torch.randint(0, 10, (16,), generator=gen), 10)
            y = y.float().to(DEV)
            prev = [t.clone() for t in params(plain)]
            mu_p, var_p = net_p.step(x, y, 0.05)
            mu_d, var_d = dp.step(x, y, 0.05)
            torch.cuda.synchronize()
            assert rel_err(mu_d, mu_p) <= 1e-5, (step, rel_err(mu_d, mu_p))
            assert rel_err(var_d, var_p) <= 1e-4, (step, rel_err(var_d, var_p))
            for i, (a, b) in enumerate(zip(params(dp_layers), params(plain))):
                if i % 2 == 0:
                    assert rel_err(a, b) <= 1e-5, (step, i, rel_err(a, b))
                else:
                    assert var_update_err(a, b, prev[i]) <= 1e-4, (step, i)
        assert dp._plan_ok and len(dp._buckets) > 1
        assert dp.peer is not None  # the SyncBN sums went through the peer exchange
        from triton_tagi._lib import lib

        assert int(lib().fn["tagi_peer_status"](1)) == 0
    finally:
        net_d.release_graph()
        torch.cuda.synchronize()
        dp.close()
