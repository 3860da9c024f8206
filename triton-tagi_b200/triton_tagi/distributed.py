"""Batch-sharded data parallelism for ``Sequential`` (one process per GPU).

The reference is single-GPU. Its update is a closed form of batch sums, so a
data-parallel step only has to combine those sums:

* forward: every BatchNorm2D all-reduces its per-channel sums
  [Σμ_z, ΣS_z, Σμ_z²] (float64) before normalising, so statistics, the Bessel
  factor and the running-stat EMA use the global batch (SyncBN);
* backward: each learnable layer writes its raw sums (aᵀδμ, (a²)ᵀδS, bias and
  γ/β sums) into a persistent buffer and an asynchronous all-reduce of that
  buffer is issued immediately; NCCL runs it on its own stream while the next
  layer's backward proceeds;
* update: after the last all-reduce the capped update is applied from the
  reduced sums on every rank with ``cap = get_cap_factor(global batch)``,
  so all replicas stay bit-identical and equal the single-batch closed form
  up to float summation order.

Only ``torch.distributed`` collectives are used, so the same code runs on
``nccl`` (GPU) and ``gloo`` (CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class DataParallel:
    """Attach to a ``Sequential``; ``net.step`` then runs data-parallel."""

    def __init__(self, net, process_group=None, sync_bn: bool = True,
                 broadcast_from: int | None = 0) -> None:
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed must be initialised before DataParallel")
        self.net = net
        self.group = process_group
        self.world_size = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self._buffers: dict[int, torch.Tensor] = {}
        self._pending: list[tuple[object, torch.Tensor, object]] = []
        net.reducer = self
        if sync_bn:
            for leaf in net.leaves():
                if hasattr(leaf, "_stats_allreduce"):  # BatchNorm2D statistics hook
                    leaf._stats_allreduce = self.allreduce_now
                    leaf._stats_world = self.world_size
        if broadcast_from is not None:
            self.broadcast_parameters(broadcast_from)

    # -- parameter synchronisation ----------------------------------------------
    def broadcast_parameters(self, src: int = 0) -> None:
        """Make every replica start from rank ``src``'s parameters."""
        for leaf in self.net.leaves():
            for name in ("mw", "Sw", "mb", "Sb", "running_mean", "running_var"):
                t = getattr(leaf, name, None)
                if t is not None:
                    if not t.is_contiguous():
                        t = t.contiguous()
                        setattr(leaf, name, t)
                    dist.broadcast(t, src=src, group=self.group)

    def allreduce_now(self, t: torch.Tensor) -> None:
        """Blocking (stream-ordered) sum over ranks, used for SyncBN statistics."""
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    # -- reducer protocol used by the layers and Sequential.step ----------------
    def begin_step(self) -> None:
        self._pending = []

    def buffer(self, layer, numel: int, dtype: torch.dtype) -> torch.Tensor:
        key = id(layer)
        buf = self._buffers.get(key)
        device = layer.mw.device
        if buf is None or buf.numel() != numel or buf.dtype != dtype or buf.device != device:
            buf = torch.empty(numel, dtype=dtype, device=device)
            self._buffers[key] = buf
        return buf

    def ready(self, layer) -> None:
        buf = self._buffers[id(layer)]
        work = dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        self._pending.append((layer, buf, work))

    def finish_step(self, cap: float) -> None:
        for layer, buf, work in self._pending:
            work.wait()
            layer._apply_sums(buf, cap)
        self._pending = []

    def step(self, x, y, sigma_v):
        return self.net.step(x, y, sigma_v)
