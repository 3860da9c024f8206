"""Data-parallel host logic on CPU with two gloo ranks.

The CUDA layers need a GPU, so these tests drive ``triton_tagi.distributed``
and ``Sequential.step`` with CPU adapter layers that implement the same
reducer protocol (``buffer`` / ``ready`` / ``_apply_sums`` and the BatchNorm
statistics hook) on top of the CPU oracle. Two ranks each take half of a
batch; afterwards both must hold the parameters of a single-process oracle
step on the whole batch (global-batch cap factor, SyncBN statistics).
"""

from __future__ import annotations

import os
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle.moments as F
from triton_tagi.base import Layer, LearnableLayer


def _rendezvous() -> str:
    """File-based rendezvous (no TCP port to race for between test runs)."""
    import tempfile

    fd, path = tempfile.mkstemp(prefix="tagi_dp_")
    os.close(fd)
    os.unlink(path)
    return f"file://{path}"


class CpuLinear(LearnableLayer):
    """Linear layer on the CPU oracle, speaking the reducer protocol."""

    def __init__(self, mw, Sw, mb, Sb):
        self.mw, self.Sw, self.mb, self.Sb = mw.clone(), Sw.clone(), mb.clone(), Sb.clone()

    num_parameters = 0

    def forward(self, ma, Sa):
        self.a = ma
        return F.mean_forward(ma, self.mw, self.mb), F.var_forward(ma, Sa, self.mw, self.Sw, self.Sb)

    def backward(self, dm, dS):
        gm, gS = F.weight_grad(self.a, dm, dS)
        K, N = self.mw.shape
        buf = self._reducer.buffer(self, 2 * (K + 1) * N, torch.float32)
        half = buf.numel() // 2
        buf[:half] = torch.cat([gm, dm.sum(0, keepdim=True)]).reshape(-1)
        buf[half:] = torch.cat([gS, dS.sum(0, keepdim=True)]).reshape(-1)
        self._reducer.ready(self)
        return F.backward_delta(dm, dS, self.mw)

    def _apply_sums(self, buf, cap):
        K, N = self.mw.shape
        half = buf.numel() // 2
        g = buf[:half].reshape(K + 1, N)
        h = buf[half:].reshape(K + 1, N)
        self.mw, self.Sw = F.capped_update(self.mw, self.Sw, self.Sw * g[:K], self.Sw**2 * h[:K], cap)
        self.mb, self.Sb = F.capped_update(self.mb, self.Sb, self.Sb * g[K:], self.Sb**2 * h[K:], cap)

    def update(self, cap):
        pass


class CpuBatchNorm(LearnableLayer):
    """BatchNorm2D on the oracle with the SyncBN statistics hook."""

    def __init__(self, C):
        self.mw, self.Sw = torch.ones(C), torch.full((C,), 1.0 / C)
        self.mb, self.Sb = torch.zeros(C), torch.full((C,), 1.0 / C)
        self.eps = 1e-5
        self._stats_allreduce, self._stats_world = None, 1

    num_parameters = 0

    def forward(self, mz, Sz):
        N, C, H, W = mz.shape
        sums = torch.stack([mz.double().sum((0, 2, 3)), Sz.double().sum((0, 2, 3)),
                            (mz.double() ** 2).sum((0, 2, 3))])
        count = N * H * W
        if self._stats_allreduce is not None:
            self._stats_allreduce(sums)
            count *= self._stats_world
        mean = (sums[0] / count).float()
        var = ((sums[1] / count).float() + (sums[2] / count).float() - mean * mean) * (count / (count - 1))
        self.var = var
        ma, Sa, self.m_hat, _ = F.bn_forward(mz, Sz, mean, var, self.mw, self.Sw, self.mb, self.Sb,
                                             self.eps)
        return ma, Sa

    def backward(self, dma, dSa):
        dmz, dSz, a, b, c, d = F.bn_backward(dma, dSa, self.m_hat, self.var, self.mw, self.eps)
        buf = self._reducer.buffer(self, 4 * self.mw.numel(), torch.float64)
        buf.copy_(torch.cat([a, b, c, d]).double())
        self._reducer.ready(self)
        return dmz, dSz

    def _apply_sums(self, buf, cap):
        a, b, c, d = buf.float().chunk(4)
        self.mw, self.Sw = F.capped_update(self.mw, self.Sw, self.Sw * a, self.Sw**2 * b, cap)
        self.mb, self.Sb = F.capped_update(self.mb, self.Sb, self.Sb * c, self.Sb**2 * d, cap)

    def update(self, cap):
        pass


class CpuReLU(Layer):
    def forward(self, mz, Sz):
        ma, Sa, self.J = F.relu_moments(mz, Sz)
        return ma, Sa

    def backward(self, dm, dS):
        return dm * self.J, dS * self.J**2


class CpuFlatten(Layer):
    def forward(self, m, S):
        self.shape = m.shape
        return m.reshape(m.shape[0], -1), S.reshape(S.shape[0], -1)

    def backward(self, dm, dS):
        return dm.reshape(self.shape), dS.reshape(self.shape)


def _make_net(seed):
    g = torch.Generator().manual_seed(seed)
    C, H, W, K1, K2 = 4, 3, 3, 36, 10
    lin1 = CpuLinear(torch.randn(K1, 16, generator=g) / 6, torch.full((K1, 16), 1 / K1),
                     torch.randn(1, 16, generator=g) * 0.1, torch.full((1, 16), 1 / K1))
    lin2 = CpuLinear(torch.randn(16, K2, generator=g) / 4, torch.full((16, K2), 1 / 16),
                     torch.randn(1, K2, generator=g) * 0.1, torch.full((1, K2), 1 / 16))
    return [CpuBatchNorm(C), CpuReLU(), CpuFlatten(), lin1, CpuReLU(), lin2]


def _data(batch=12):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(batch, 4, 3, 3, generator=g) + 0.5
    y = torch.nn.functional.one_hot(torch.randint(0, 10, (batch,), generator=g), 10).float()
    return x, y


def _worker(rank, world, init, out_q, bucket_bytes=4 << 20, steps=2):
    import datetime

    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        import triton_tagi.network as net_mod
        from triton_tagi.distributed import DataParallel

        # Sequential.step calls the CUDA innovation kernel; use the oracle's on CPU.
        net_mod.compute_innovation = lambda y, mu, var, sv: F.innovation(y, mu, var, sv)
        net = net_mod.Sequential(_make_net(0), device="cpu")
        dp = DataParallel(net, broadcast_from=0, bucket_bytes=bucket_bytes)
        x, y = _data()
        shard = x.shape[0] // world
        sl = slice(rank * shard, (rank + 1) * shard)
        for _ in range(steps):
            dp.step(x[sl], y[sl], 0.05)
        if steps > 1:  # buckets planned after the first step
            assert dp._plan_ok and len(dp._buckets) >= 1
        # numpy arrays travel by value: a torch tensor would travel as a shared-memory
        # handle that is gone if this process exits before the parent receives it
        out_q.put((rank, [t.clone().numpy() for l in net.leaves() for t in (l.mw, l.Sw, l.mb, l.Sb)]))
    finally:
        dist.destroy_process_group()


def _single_process_reference(steps=2):
    """Full-batch steps with the plain oracle (same maths, no sharding)."""
    layers = _make_net(0)
    x, y = _data()

    class Red:
        world_size = 1

        def __init__(self):
            self.bufs, self.pending = {}, []

        def buffer(self, layer, n, dt):
            self.bufs[id(layer)] = torch.empty(n, dtype=dt)
            return self.bufs[id(layer)]

        def ready(self, layer):
            self.pending.append(layer)

        def begin_step(self):
            self.pending = []

        def finish_step(self, cap):
            for layer in self.pending:
                layer._apply_sums(self.bufs[id(layer)], cap)

    red = Red()
    for _ in range(steps):
        m, S = x, torch.zeros_like(x)
        for layer in layers:
            m, S = layer.forward(m, S)
        dm, dS = F.innovation(y, m, S, 0.05)
        cap = F.get_cap_factor(x.shape[0])
        for layer in layers:
            if hasattr(layer, "_set_param_mode"):
                layer._set_param_mode("sums", cap, red)
        red.begin_step()
        for layer in reversed(layers):
            dm, dS = layer.backward(dm, dS)
        red.finish_step(cap)
    return [t for l in layers if hasattr(l, "_apply_sums") for t in (l.mw, l.Sw, l.mb, l.Sb)]


@pytest.mark.parametrize("bucket_bytes,steps", [(4 << 20, 2), (600, 3)])
def test_two_rank_step_equals_full_batch_step(bucket_bytes, steps):
    """Two ranks, each half of the batch, equal the full-batch step; the first
    step all-reduces every layer's buffer on its own, later steps go through
    the buckets (one bucket per dtype, or with 600-byte buckets one per layer
    group that fits)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init = _rendezvous()
    procs = [ctx.Process(target=_worker, args=(r, 2, init, q, bucket_bytes, steps))
             for r in range(2)]
    for p in procs:
        p.start()
    results = {r: [torch.from_numpy(a) for a in arrs]
               for r, arrs in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = _single_process_reference(steps)
    for r in (0, 1):
        for got, want in zip(results[r], ref):
            torch.testing.assert_close(got, want, rtol=2e-5, atol=1e-7)
    for a, b in zip(results[0], results[1]):  # replicas stay identical
        assert torch.equal(a, b)


def _leaver(rank, world, init, out_q):
    import datetime

    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)  # one healthy collective
    if rank == 1:
        out_q.put((rank, "left"))
        out_q.close()
        out_q.join_thread()
        os._exit(0)  # leaves between steps, before the next collective
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)
        out_q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - the timeout type differs across versions
        out_q.put((rank, f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}"))


def test_rank_that_leaves_is_detected_by_bounded_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init = _rendezvous()
    procs = [ctx.Process(target=_leaver, args=(r, 2, init, q)) for r in range(2)]
    for p in procs:
        p.start()
    msgs = dict(q.get(timeout=60) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert msgs[1] == "left"
    assert msgs[0].startswith("error"), msgs[0]
