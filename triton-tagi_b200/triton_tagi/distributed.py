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

Buckets: the first step records the order (and dtype) in which the layers
request their sum buffers, which is the order in which they become ready.
From then on every buffer is a view into a flat bucket of at most
``bucket_bytes`` (one dtype per bucket; a larger buffer is a bucket of its
own), and one all-reduce is issued per bucket when its last layer is ready:
the 20 BatchNorm γ/β buffers of a ResNet-18 (a few KB each, float64) travel
as one message instead of twenty, and the small convolutions of the early
stages are grouped the same way.

SyncBN statistics: with the nccl backend, on one host with peer access between
all GPUs, the 3·C float64 sums go through ``PeerExchange`` (one kernel over
NVLink peer memory, a few microseconds) instead of an NCCL all-reduce (tens
of microseconds at eight GPUs, twenty times per ResNet-18 step, each on the
critical path); ``close()`` releases its buffers.

``timer`` (optional): a callable ``timer(phase, what)`` with phase "before" /
"after" around each SyncBN statistics all-reduce (what = "syncbn"), each wait
for a bucket's all-reduce at the end of the backward ("grad_wait") and the
application of the reduced sums ("apply"); the benchmark records CUDA events
there.

Only ``torch.distributed`` collectives are used, so the same code runs on
``nccl`` (GPU) and ``gloo`` (CPU tests).
"""

from __future__ import annotations

import ctypes
import socket

import torch
import torch.distributed as dist

from ._lib import lib, stream


class PeerExchange:
    """All-reduce of small float64 vectors through NVLink peer memory
    (``tagi_peer_allreduce_f64``): every rank stores its values into every
    rank's exchange buffer, raises a flag, waits for all flags and adds the
    slots in rank order. One kernel, no collective library, replayable from a
    CUDA graph; used for the SyncBN statistics (3·C doubles), whose all-reduce
    sits on the critical path of every data-parallel BatchNorm2D.

    Built only when every rank runs on one host and its GPU can reach every
    other rank's GPU (``available``); buffers are exchanged as CUDA IPC
    handles. Vectors longer than ``max_elems`` are not handled here."""

    def __init__(self, group, rank: int, world: int, device, max_elems: int = 4096) -> None:
        L = lib()
        self.rank, self.world, self.max_elems = rank, world, max_elems
        self.device = torch.device(device)
        nbytes = L.size("tagi_peer_buffer_bytes", world, max_elems)
        handle = ctypes.create_string_buffer(64)
        own = ctypes.c_void_p()
        L("tagi_peer_buffer_create", nbytes, ctypes.addressof(own), handle)
        self._own = own.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        self._opened, ptrs = [], []
        for r in range(world):
            if r == rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            L("tagi_peer_buffer_open", ctypes.create_string_buffer(handles[r], 64),
              ctypes.addressof(p))
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.counter = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.group = group
        dist.barrier(group=group)  # every rank's buffers are open before any exchange

    @staticmethod
    def available(group, device) -> bool:
        """True if all ranks share this host and this GPU reaches every other
        rank's GPU (collective: every rank must call it)."""
        dev = torch.device(device)
        info = [None] * dist.get_world_size(group)
        dist.all_gather_object(info, (socket.gethostname(), dev.index), group=group)
        if len({h for h, _ in info}) != 1:
            return False
        ok = all(d == dev.index or torch.cuda.can_device_access_peer(dev.index, d)
                 for _, d in info)
        flags = [None] * len(info)
        dist.all_gather_object(flags, ok, group=group)
        return all(flags)

    def allreduce(self, t: torch.Tensor) -> None:
        lib()("tagi_peer_allreduce_f64", t.data_ptr(), t.numel(), self.table.data_ptr(),
              self.rank, self.world, self.max_elems, self.counter.data_ptr(), stream(t))

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        L = lib()
        for p in self._opened:
            L("tagi_peer_buffer_close", p, 0)
        dist.barrier(group=self.group)
        L("tagi_peer_buffer_close", self._own, 1)
        self._own, self._opened = None, []


class DataParallel:
    """Attach to a ``Sequential``; ``net.step`` then runs data-parallel."""

    def __init__(self, net, process_group=None, sync_bn: bool = True,
                 broadcast_from: int | None = 0, bucket_bytes: int = 4 << 20,
                 capturable: bool = False, peer_stats: bool | None = None) -> None:
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed must be initialised before DataParallel")
        if capturable and dist.get_backend(process_group) != "nccl":
            raise ValueError("DataParallel(capturable=True) needs the nccl backend")
        # Sequential(cuda_graph=True) may capture the data-parallel step (with its
        # collectives) into a CUDA graph; release it (net.release_graph()) before
        # the process group is destroyed.
        self.capturable = capturable
        self.net = net
        self.group = process_group
        self.world_size = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self.bucket_bytes = bucket_bytes
        self.timer = None
        self._buffers: dict[int, torch.Tensor] = {}  # layer -> its own buffer (first step)
        self._order: list[tuple] = []                # (key, layer, numel, dtype, device)
        self._views: dict[int, torch.Tensor] = {}    # layer -> view into a bucket
        self._bucket_of: dict[int, int] = {}
        self._buckets: list[dict] = []               # flat tensor + member layers
        self._pending: list[tuple[list, torch.Tensor, object]] = []
        self._left: list[int] = []
        self._plan_ok = False
        net.reducer = self
        # SyncBN statistics through NVLink peer memory (nccl backend, one host,
        # peer access everywhere); otherwise through the collective library
        self.peer = None
        if peer_stats is None:
            peer_stats = sync_bn and dist.get_backend(process_group) == "nccl"
        if peer_stats:
            dev = net.device if net.device.index is not None else torch.device(
                "cuda", torch.cuda.current_device())
            if PeerExchange.available(process_group, dev):
                self.peer = PeerExchange(process_group, self.rank, self.world_size, dev)
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

    def _time(self, phase: str, what: str) -> None:
        if self.timer is not None:
            self.timer(phase, what)

    def allreduce_now(self, t: torch.Tensor) -> None:
        """Blocking (stream-ordered) sum over ranks, used for SyncBN statistics."""
        self._time("before", "syncbn")
        if (self.peer is not None and t.dtype == torch.float64 and t.is_contiguous()
                and t.numel() <= self.peer.max_elems):
            self.peer.allreduce(t)
        else:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        self._time("after", "syncbn")

    def close(self) -> None:
        """Release the peer exchange buffers (collective; before the process
        group is destroyed, after any CUDA graph that uses them)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    # -- reducer protocol used by the layers and Sequential.step ----------------
    def begin_step(self) -> None:
        self._pending = []
        self._order = []
        self._left = [len(b["layers"]) for b in self._buckets]

    def buffer(self, layer, numel: int, dtype: torch.dtype) -> torch.Tensor:
        key = id(layer)
        device = layer.mw.device
        self._order.append((key, layer, numel, dtype, device))
        view = self._views.get(key) if self._plan_ok else None
        if view is not None and view.numel() == numel and view.dtype == dtype \
                and view.device == device:
            return view
        self._plan_ok = False  # a new layer or a new size: plan again after this step
        buf = self._buffers.get(key)
        if buf is None or buf.numel() != numel or buf.dtype != dtype or buf.device != device:
            buf = torch.empty(numel, dtype=dtype, device=device)
            self._buffers[key] = buf
        return buf

    def _issue(self, layers: list, flat: torch.Tensor) -> None:
        work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        self._pending.append((layers, flat, work))

    def ready(self, layer) -> None:
        key = id(layer)
        if self._plan_ok and key in self._bucket_of:
            b = self._bucket_of[key]
            self._left[b] -= 1
            if self._left[b] == 0:
                bucket = self._buckets[b]
                self._issue(bucket["layers"], bucket["flat"])
            return
        self._issue([layer], self._buffers[key])

    def finish_step(self, cap: float) -> None:
        if self._plan_ok and any(n != 0 for n in self._left):
            raise RuntimeError("DataParallel: a bucket's layers did not all report ready")
        for _, _, work in self._pending:
            self._time("before", "grad_wait")
            work.wait()
            self._time("after", "grad_wait")
        self._time("before", "apply")
        for layers, _, _ in self._pending:
            for layer in layers:
                key = id(layer)
                buf = self._views[key] if self._plan_ok and key in self._views \
                    else self._buffers[key]
                layer._apply_sums(buf, cap)
        self._time("after", "apply")
        self._pending = []
        if not self._plan_ok:
            self._plan()

    def _plan(self) -> None:
        """Group this step's buffers, in the order they were requested, into
        buckets of one dtype and at most ``bucket_bytes`` each; a bucket's
        members keep the order in which they become ready."""
        self._buckets, self._views, self._bucket_of = [], {}, {}
        open_by: dict = {}
        align = 64  # elements: every view starts 256-byte aligned
        groups: list[dict] = []
        for key, layer, numel, dtype, device in self._order:
            esize = torch.empty((), dtype=dtype).element_size()
            size = (numel + align - 1) // align * align
            g = open_by.get((dtype, device))
            if g is None or (g["elems"] + size) * esize > self.bucket_bytes:
                g = {"dtype": dtype, "device": device, "members": [], "elems": 0}
                groups.append(g)
                open_by[(dtype, device)] = g
            g["members"].append((key, layer, numel, g["elems"]))
            g["elems"] += size
        for i, g in enumerate(groups):
            flat = torch.zeros(g["elems"], dtype=g["dtype"], device=g["device"])
            self._buckets.append({"flat": flat,
                                  "layers": [layer for _, layer, _, _ in g["members"]]})
            for key, _, numel, off in g["members"]:
                self._views[key] = flat[off:off + numel]
                self._bucket_of[key] = i
        self._buffers = {}
        self._plan_ok = True

    def step(self, x, y, sigma_v):
        return self.net.step(x, y, sigma_v)
