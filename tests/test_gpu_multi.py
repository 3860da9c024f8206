"""Multi-GPU checks (skipped with fewer than two GPUs).

* The NVLink peer-memory all-reduce of the SyncBN statistics
  (``PeerExchange``, ``tagi_peer_allreduce_f64``): two ranks, one process per
  GPU, reduce vectors of several lengths, eagerly and replayed from a CUDA
  graph; every rank must get the sum in rank order, bit-identical across ranks.
* A two-rank data-parallel ResNet step (reduced width) against the same network
  stepped on one GPU with the whole batch: predictions and parameters agree at
  the parity bar, and the replicas are bit-identical.
"""

from __future__ import annotations

import datetime
import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _need_two():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def _init(rank, world, path):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{path}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))


def _exchange_worker(rank, world, path, q):
    import sys

    sys.path[:0] = [os.path.join(os.path.dirname(__file__), ".."),
                    os.path.join(os.path.dirname(__file__), "..", "triton-tagi_b200")]
    _init(rank, world, path)
    try:
        from triton_tagi._lib import lib
        from triton_tagi.distributed import PeerExchange

        dev = torch.device("cuda", rank)
        assert PeerExchange.available(None, dev)
        px = PeerExchange(None, rank, world, dev, max_elems=2048)
        out = []
        g = torch.Generator().manual_seed(100 + rank)
        for n in (1, 7, 192, 1536, 2048):
            mine = torch.randn(n, generator=g, dtype=torch.float64).to(dev)
            allv = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allv, mine)
            want = torch.zeros_like(mine)
            for v in allv:
                want += v
            t = mine.clone()
            px.allreduce(t)
            torch.cuda.synchronize()
            out.append(bool(torch.equal(t, want)))
        # replayed from a CUDA graph (the epoch counter lives on the device)
        buf = torch.zeros(512, dtype=torch.float64, device=dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            px.allreduce(buf)
        for rep in range(3):
            vals = torch.full((512,), float(rank + 1 + rep), dtype=torch.float64, device=dev)
            buf.copy_(vals)
            graph.replay()
            torch.cuda.synchronize()
            want = sum(float(r + 1 + rep) for r in range(world))
            out.append(bool(torch.all(buf == want).item()))
        del graph
        torch.cuda.synchronize()
        out.append(int(lib().fn["tagi_peer_status"](1)) == 0)
        px.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def _run(target, world=2):
    fd, path = tempfile.mkstemp(prefix="tagi_nccl2_")
    os.close(fd)
    os.unlink(path)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, path, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_peer_exchange_two_ranks():
    _need_two()
    res = _run(_exchange_worker)
    for rank, flags in res.items():
        assert all(flags), (rank, flags)


def _dp_worker(rank, world, path, q):
    import sys

    sys.path[:0] = [os.path.dirname(__file__), os.path.join(os.path.dirname(__file__), ".."),
                    os.path.join(os.path.dirname(__file__), "..", "triton-tagi_b200")]
    _init(rank, world, path)
    try:
        import triton_tagi as TT
        from _nets import build_config, params
        from triton_tagi.distributed import DataParallel

        dev = torch.device("cuda", rank)
        torch.manual_seed(5)
        layers = build_config("r18", TT, device=dev, width=0.25)
        net = TT.Sequential(layers, device=dev, cuda_graph=True)
        dp = DataParallel(net, capturable=True)
        gen = torch.Generator().manual_seed(11)
        B = 16
        for _ in range(3):
            x = torch.randn(B * world, 3, 32, 32, generator=gen)
            y = torch.nn.functional.one_hot(torch.randint(0, 10, (B * world,), generator=gen), 10)
            sl = slice(rank * B, (rank + 1) * B)
            mu, var = dp.step(x[sl].to(dev), y[sl].float().to(dev), 0.05)
        torch.cuda.synchronize()
        q.put((rank, (mu.cpu().numpy(), var.cpu().numpy(),
                      [t.detach().cpu().numpy() for t in params(layers)])))
        net.release_graph()
        torch.cuda.synchronize()
        dp.close()
    finally:
        dist.destroy_process_group()


def test_two_rank_step_equals_one_gpu_global_batch():
    _need_two()
    import triton_tagi as TT
    from _nets import build_config, params
    from _tol import rel_err, var_update_err

    res = _run(_dp_worker)
    # the same three steps on one GPU over the whole batch
    dev = torch.device("cuda", 0)
    torch.manual_seed(5)
    layers = build_config("r18", TT, device=dev, width=0.25)
    init = [t.detach().clone() for t in params(layers)]
    net = TT.Sequential(layers, device=dev)
    gen = torch.Generator().manual_seed(11)
    B, world = 16, 2
    for _ in range(3):
        x = torch.randn(B * world, 3, 32, 32, generator=gen)
        y = torch.nn.functional.one_hot(torch.randint(0, 10, (B * world,), generator=gen), 10)
        mu, var = net.step(x.to(dev), y.float().to(dev), 0.05)
    ref = [t.detach().cpu() for t in params(layers)]
    for r in range(world):
        mu_r, var_r, prm = res[r]
        assert rel_err(mu_r, mu[r * B:(r + 1) * B]) <= 1e-4
        assert rel_err(var_r, var[r * B:(r + 1) * B]) <= 1e-3
        for i, (a, b) in enumerate(zip(prm, ref)):
            if i % 2 == 0:
                assert rel_err(a, b) <= 1e-4, (r, i, rel_err(a, b))
            else:
                assert var_update_err(a, b, init[i]) <= 1e-3, (r, i)
    for a, b in zip(res[0][2], res[1][2]):
        assert (a == b).all()
