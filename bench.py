"""Benchmark of the TAGI training step (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload r18|mlp|cnn|tfm]
                    [--impl ours|reference]

Default workload: the ResNet-18 configuration (3×32×32 N(0,1) inputs, 128 per
GPU, gain 0.1, σ_v = 0.05, one-hot labels over 10 classes), one
``Sequential.step`` (forward + innovation + backward + capped update) per
step, batch-sharded over N GPUs (weak scaling, one process per GPU, launched
by torchrun for N > 1).

value      samples/s over all ranks: K·B·N / (max over ranks of the summed
           CUDA-event step times), inputs resident in HBM, L2 flushed
           (256 MiB write) before every step outside the timed events.
e2e        the same metric through the public API with pinned host buffers:
           H2D of x, y and D2H of (μ, S) inside the timed events.
roofline   the dominant moment contraction, timed with CUDA events around
           each of its launches in up to 3 steps after the timed ones; achieved
           = algorithmic FLOPs (6·M·N·K forward, 4·M·N·K backward/weight sums)
           ÷ time, against the 3xTF32-effective tensor peak (measured cuBLAS
           TF32 ÷ 3). One GPU with a captured step: the events are nodes of a
           second capture of the step, replayed (no host launch gaps inside the
           intervals); otherwise eager steps (`entry_timing` says which).
cpu_baseline  the CPU oracle (float32 PyTorch restatement of the reference's
           equations) on the host cores, rank 0 at N = 1, at the workload's
           own batch (5 timed steps after 1 warm-up).
subrecords the MLP step at the same number of GPUs, and on one GPU the Linear
           sweep's 8192 x 4096 x 4096 shape (forward, input deltas, weight
           sums + capped update), from the same run.
clocks     SM clock (median, min) and the clock-event reasons seen, read
           through NVML every 10 ms during the timed steps (read-only).
device_status  the tensor-core kernels' error word after the timed steps
           (non-zero: a bounded wait ran out; the run then exits with an error).
replicas_bit_identical  (N > 1) every rank's parameters after the run have the
           same bits.
--impl reference  times that CPU restatement as the reference arm, at the
           workload's own batch.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (str(ROOT), str(ROOT / "triton-tagi_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

SIGMA_V = 0.05
_NETS: list = []  # networks whose CUDA graphs are released before the process group
WORKLOADS = {
    "r18": dict(batch=128, metric="TAGI ResNet-18 Sequential.step samples/sec"),
    "mlp": dict(batch=256, metric="TAGI MLP 784-256-128-10 Sequential.step samples/sec"),
    "cnn": dict(batch=512, metric="TAGI CNN Sequential.step samples/sec"),
    "tfm": dict(batch=32, metric="TAGI transformer Sequential.step samples/sec"),
    "swp": dict(batch=8192, metric="TAGI Linear op sweep: fused mean/var moment GEMM TFLOP/s"),
}
SWEEP = [(m, k) for m in (256, 1024, 4096, 8192) for k in (1024, 4096)]


# ----------------------------------------------------------------------------- networks
def build_layers(name: str, L, device):
    d = dict(device=device)
    if name == "mlp":
        return [L.Linear(784, 256, **d), L.ReLU(), L.Linear(256, 128, **d), L.ReLU(),
                L.Linear(128, 10, **d), L.Remax()]
    if name == "cnn":
        return [L.Conv2D(3, 32, 5, padding=2, **d), L.ReLU(), L.AvgPool2D(2),
                L.Conv2D(32, 64, 5, padding=2, **d), L.BatchNorm2D(64, **d), L.ReLU(),
                L.AvgPool2D(2), L.Conv2D(64, 64, 5, padding=2, **d), L.ReLU(), L.AvgPool2D(2),
                L.Flatten(), L.Linear(1024, 256, **d), L.ReLU(), L.Linear(256, 10, **d),
                L.Remax()]
    if name == "r18":
        kw = dict(gain_w=0.1, gain_b=0.1, **d)
        return [L.Conv2D(3, 64, 3, stride=1, padding=1, **kw), L.ReLU(), L.BatchNorm2D(64, **kw),
                L.ResBlock(64, 64, 1, **kw), L.ResBlock(64, 64, 1, **kw),
                L.ResBlock(64, 128, 2, **kw), L.ResBlock(128, 128, 1, **kw),
                L.ResBlock(128, 256, 2, **kw), L.ResBlock(256, 256, 1, **kw),
                L.ResBlock(256, 512, 2, **kw), L.ResBlock(512, 512, 1, **kw),
                L.AvgPool2D(4), L.Flatten(), L.Linear(512, 10, **kw), L.Remax()]
    if name == "tfm":
        V, E, H, S = 64, 512, 8, 512
        layers = [L.Embedding(V, E, input_size=S, scale=0.25, **d), L.PositionalEncoding(E, **d)]
        for _ in range(4):
            layers += [L.MultiheadAttentionV2(E, H, S, bias=False, **d), L.RMSNorm(E, **d),
                       L.Linear(E, 4 * E, **d), L.ReLU(), L.Linear(4 * E, E, **d)]
        return layers + [L.Linear(E, V, **d)]
    raise KeyError(name)


def make_batch(name: str, batch: int, seed: int, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    if name == "mlp":
        x = torch.randn(batch, 784, generator=g)
    elif name == "tfm":
        x = torch.randint(0, 64, (batch, 512), generator=g).float()
    else:
        x = torch.randn(batch, 3, 32, 32, generator=g)
    if name == "tfm":
        y = torch.nn.functional.one_hot(torch.flip(x.long(), dims=[1]), 64).float()
    else:
        y = torch.nn.functional.one_hot(torch.randint(0, 10, (batch,), generator=g), 10).float()
    return x.to(device), y.to(device)


# ----------------------------------------------------------------------------- helpers
class ClockSampler:
    """SM clock and clock-event (throttle) reasons read through NVML every
    ``period`` seconds while the timed region runs. Read-only: no setting of the
    GPU is touched. The first sample is taken before ``__enter__`` returns, so a
    timed region of a few hundred milliseconds still carries tens of samples."""

    # NVML clock-event reason bits reported (nvmlClocksEventReason*)
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))

    def __init__(self, index: int, period: float = 0.01):
        self.index, self.period = index, period
        self.sm, self.power, self.max_sm, self.mask = [], [], None, 0
        self.error, self._nvml, self._thread = None, None, None
        self._stop = threading.Event()

    def _handle(self, nv):
        try:  # CUDA and NVML may order devices differently: match the PCI address
            p = torch.cuda.get_device_properties(self.index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def _sample(self):
        nv, h = self._nvml, self._h
        self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
        self.mask |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
        try:
            self.power.append(nv.nvmlDeviceGetPowerUsage(h) / 1e3)
        except Exception:
            pass

    def _loop(self):
        while not self._stop.wait(self.period):
            try:
                self._sample()
            except Exception as e:  # keep what was sampled so far
                self.error = repr(e)
                return

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = self._handle(pynvml)
            self.max_sm = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
            self._sample()
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
        except Exception as e:
            self.error = repr(e)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2.0)
            try:  # a region shorter than the period is still bracketed by two samples
                self._sample()
            except Exception as e:
                self.error = repr(e)
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        d = {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_sm,
             "samples": len(self.sm),
             "reasons": sorted(n for n, bit in self.REASONS if self.mask & bit),
             "source": "nvml", "period_ms": 1e3 * self.period}
        if self.sm:
            d["sm_mhz_min"] = min(self.sm)
        if self.power:
            d["power_w_median"] = round(statistics.median(self.power), 1)
        if self.error:
            d["error"] = self.error
        return d


def _conv_pixels(a) -> int:
    """Ho*Wo of a tagi_conv2d_forward call (H, W, k, stride, padding, padding_type
    at argument positions 10, 11, 13, 14, 15, 16)."""
    H, W, k, s, p, pt = a[10], a[11], a[13], a[14], a[15], a[16]
    if pt == 2 and p > 0:
        return ((H + p - k) // s + 1) * ((W + p - k) // s + 1)
    return ((H + 2 * p - k) // s + 1) * ((W + 2 * p - k) // s + 1)


def _out_pixels(H, W, k, s, p, pt) -> int:
    if pt == 2 and p > 0:
        return ((H + p - k) // s + 1) * ((W + p - k) // s + 1)
    return ((H + 2 * p - k) // s + 1) * ((W + 2 * p - k) // s + 1)


def _planes(*ptrs) -> int:
    return sum(1 for q in ptrs if q)


# Algorithmic HBM bytes of the memory-bound library entries (each input element
# read once, each output element written once).
ENTRY_BYTES = {
    "tagi_relu_forward": lambda a: 20 * a[5],
    "tagi_jacobian_backward": lambda a: 20 * a[5],
    "tagi_innovation": lambda a: 20 * a[5],
    "tagi_add_inplace": lambda a: 24 * a[4],
    "tagi_capped_update": lambda a: 24 * a[4],
    "tagi_remax_forward": lambda a: 20 * a[5] * a[6],
    # ids read, rows written (mean and variance)
    "tagi_embedding_forward": lambda a: (4 + 8 * a[7]) * a[5],
    "tagi_positional_add": lambda a: 8 * a[3] * a[5],
    "tagi_bn_channel_sums": lambda a: 8 * a[3] * a[4] * a[5],
    # reads mz, Sz; writes ma, Sa, m_hat
    "tagi_bn_train_forward": lambda a: (20 + 8 * _planes(a[13])) * a[15] * a[16] * a[17],
    "tagi_bn_forward": lambda a: 4 * (5 + _planes(a[11])) * a[12] * a[13] * a[14],
    "tagi_bn_backward": lambda a: (24 if a[7] else 20) * a[10] * a[11] * a[12],
    "tagi_avgpool_forward": lambda a: 8 * a[4] * a[5] * a[6] * a[7] * (1 + 1 / a[8] ** 2),
    "tagi_avgpool_backward": lambda a: 8 * a[4] * a[5] * a[6] * a[7] * (1 + 1 / a[8] ** 2),
    # patches written (mean, and variance if given) + image read
    "tagi_im2col": lambda a: 4 * _planes(a[0], a[1]) * a[4] * a[5] * (
        a[6] * a[7] + _out_pixels(a[6], a[7], a[8], a[9], a[10], a[11]) * a[8] * a[8]),
    "tagi_im2col_t": lambda a: 4 * a[2] * a[3] * (
        a[4] * a[5] + _out_pixels(a[4], a[5], a[6], a[7], a[8], a[9]) * a[6] * a[6]),
    "tagi_nchw_to_nhwc": lambda a: 8 * _planes(a[0], a[1]) * a[4] * a[5] * a[6],
    "tagi_col2im": lambda a: 8 * a[4] * a[5] * (
        a[6] * a[7] + _out_pixels(a[6], a[7], a[8], a[9], a[10], a[11]) * a[8] * a[8]),
}


# DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum) of the
# contraction families. r18: the family averages of a batch-64 capture of one
# step's 59 tensor-core launches (the stem's weight sums and the classifier run
# on CUDA cores), doubled for batch 128; a later single-launch full capture of
# the forward family's stage-2 convolution gave 32.2 MB at batch 64 (64.4 MB
# doubled), in line with the forward average. swp: one 4096 x 4096 x 4096 Linear
# forward scaled by M to the sweep's 8192-row headline (A and the number of B
# re-reads both grow with M).
MEASURED_TRAFFIC = {
    ("r18", "moment_forward"): 63.1e6,
    ("r18", "backward_delta"): 37.4e6,
    ("r18", "param_grad"): 157.2e6,
    ("swp", "moment_forward"): 2 * 1.833e9,
}


class LaunchTimer:
    """Times every library call with CUDA events (library call hook): the moment
    contractions by family with their flops, the other entries by name with
    their algorithmic bytes where known."""

    FAMILIES = {
        "tagi_moment_forward": ("moment_forward", lambda a: 6.0 * a[17] * a[18] * a[19]),
        # M = N*Ho*Wo output pixels, N = Co, reduction C*k*k
        "tagi_conv2d_forward": ("moment_forward", lambda a: 6.0 * a[8] * _conv_pixels(a) * a[12]
                                * a[9] * a[13] * a[13]),
        "tagi_backward_delta_view": ("backward_delta", lambda a: 4.0 * a[14] * a[15] * a[16]),
        "tagi_fused_backward_delta": ("backward_delta", lambda a: 4.0 * a[5] * a[6] * a[7]),
        "tagi_linear_forward": ("moment_forward", lambda a: 6.0 * a[8] * a[9] * a[10]),
        "tagi_linear_backward_delta": ("backward_delta", lambda a: 4.0 * a[5] * a[6] * a[7]),
        # M = N*H*W input pixels, N = C, reduction Co*k*k
        # (args: dmz, dSz, mw, d_ma, d_Sa, N, C, H, W, Co, k, stride, padding, ...)
        "tagi_conv2d_backward_delta": (
            "backward_delta", lambda a: 4.0 * a[5] * a[7] * a[8] * a[6] * a[9] * a[10] * a[10]),
        "tagi_param_grad": ("param_grad", lambda a: 4.0 * a[8] * a[9] * a[10]),
        "tagi_param_grad_t": ("param_grad", lambda a: 4.0 * a[8] * a[9] * a[10]),
        "tagi_param_grad_bias_given": ("param_grad", lambda a: 4.0 * a[9] * a[10] * a[11]),
    }

    def __init__(self, external: bool = False):
        # external: the events become event-record nodes of a CUDA graph being
        # captured, so every replay times the same calls again
        self.records, self._open, self.external = [], None, external
        self.seconds, self.reps = None, 0

    def __call__(self, phase, name, args):
        ev = torch.cuda.Event(enable_timing=True, external=self.external)
        ev.record()
        if phase == "before":
            self._open = ev
            return
        fam = self.FAMILIES.get(name)
        if fam is not None:
            self.records.append((fam[0], fam[1](args), None, self._open, ev))
        else:
            nb = ENTRY_BYTES.get(name)
            self.records.append((name, None, nb(args) if nb else None, self._open, ev))

    def harvest(self):
        """Adds every recorded call's event interval (after a synchronize): once
        after eager steps, or after each replay of a captured step."""
        if self.seconds is None:
            self.seconds = [0.0] * len(self.records)
        for i, (_, _, _, a, b) in enumerate(self.records):
            self.seconds[i] += a.elapsed_time(b) * 1e-3
        self.reps += 1

    def summary(self):
        """(contraction families, other entries), over every harvested pass."""
        if self.seconds is None:
            self.harvest()
        fam, other = {}, {}
        for (name, flops, nbytes, _, _), t in zip(self.records, self.seconds):
            d = fam if flops is not None else other
            f = d.setdefault(name, {"launches": 0, "flops": 0.0, "bytes": 0.0, "seconds": 0.0,
                                    "bytes_known": True})
            f["launches"] += self.reps
            f["flops"] += self.reps * (flops or 0.0)
            f["bytes"] += self.reps * (nbytes or 0.0)
            f["bytes_known"] &= nbytes is not None
            f["seconds"] += t
        return fam, other


class CollectiveTimer:
    """CUDA events around the data-parallel reducer's collectives (its timer hook)."""

    def __init__(self):
        self.open, self.records = {}, []

    def __call__(self, phase, what):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        if phase == "before":
            self.open[what] = ev
        else:
            self.records.append((what, self.open.pop(what), ev))

    def summary(self, steps: int) -> dict:
        torch.cuda.synchronize()
        out = {}
        for what, a, b in self.records:
            d = out.setdefault(what, {"calls_per_step": 0.0, "ms_per_step": 0.0})
            d["calls_per_step"] += 1.0 / steps
            d["ms_per_step"] += a.elapsed_time(b) / steps
        return out


def tf32_peak_tflops(device) -> float:
    """Burst cuBLAS TF32 throughput on an 8192³ GEMM: the median of 9 single
    launches timed with CUDA events after 3 warm-up launches (the best of a few
    moved by ±5 % between runs)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        n = 8192
        a = torch.randn(n, n, device=device)
        b = torch.randn(n, n, device=device)
        for _ in range(3):
            torch.matmul(a, b)
        times = []
        for _ in range(9):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch.matmul(a, b)
            e.record()
            e.synchronize()
            times.append(s.elapsed_time(e) * 1e-3)
        del a, b
        return 2.0 * n**3 / statistics.median(times) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            pass
    return {}


# ----------------------------------------------------------------------------- CPU arms
def cpu_rate(workload: str, steps: int, warmup: int, budget_s: float) -> dict:
    """Samples/s of the CPU oracle (float32 PyTorch on all host threads) at the
    workload's own batch. Only if (steps + warmup) steps at that batch would
    take much longer than ``budget_s`` (a slow host) is the batch reduced; the
    sample string says which batch was timed."""
    import oracle.net as ON

    torch.set_num_threads(os.cpu_count() or 1)
    full = WORKLOADS[workload]["batch"]
    torch.manual_seed(0)
    net = ON.Sequential(build_layers(workload, ON, "cpu"))
    probe_b = min(full, 16)
    x, y = make_batch(workload, probe_b, 1)
    t0 = time.perf_counter()
    net.step(x, y, SIGMA_V)
    per_sample = (time.perf_counter() - t0) / probe_b
    target = 2.0 * budget_s / max(1, steps + warmup)
    batch = full if per_sample * full <= target else int(max(2, target / max(per_sample, 1e-6)))
    x, y = make_batch(workload, batch, 2)
    for _ in range(warmup):
        net.step(x, y, SIGMA_V)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        net.step(x, y, SIGMA_V)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    return {"value": steps * batch / total, "unit": "samples/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{workload} Sequential.step at batch {batch} (of {full}),"
                      f" {steps} timed steps after {warmup} warm-up, float32 oracle on "
                      f"{torch.get_num_threads()} threads",
            "batch": batch, "ms_per_step": 1e3 * total / steps}


def reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    r = cpu_rate(args.workload, args.steps, args.warmup, budget_s=150.0)
    line = {
        "impl": "reference", "metric": WORKLOADS[args.workload]["metric"], "value": r["value"],
        "unit": "samples/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        # our arm's workload configuration; the bounded sample actually timed is
        # described in cpu_baseline.sample
        "config": {"workload": args.workload, "batch_per_gpu": WORKLOADS[args.workload]["batch"],
                   "global_batch": WORKLOADS[args.workload]["batch"] * world,
                   "sigma_v": SIGMA_V, "parallelism": f"dp{world}"},
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": r["value"], "unit": "samples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def our_arm(args, rank: int, world: int, local: int) -> None:
    import triton_tagi as TT
    from triton_tagi._lib import device_status, kernel_launches, lib

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B = WORKLOADS[args.workload]["batch"]
    torch.manual_seed(1234)
    # Steps of small networks are a few dozen short kernels: replay them from a
    # CUDA graph (Sequential(cuda_graph=True)); the data-parallel step is captured
    # with its NCCL collectives (--no-dp-graph: eager).
    graphed = args.workload in ("mlp", "cnn", "r18") and not args.no_graph and (
        world == 1 or args.dp_graph)
    net = TT.Sequential(build_layers(args.workload, TT, dev), device=dev, cuda_graph=graphed)
    _NETS.append(net)
    if world > 1:
        from triton_tagi.distributed import DataParallel

        DataParallel(net, capturable=args.dp_graph)
    x, y = make_batch(args.workload, B, 100 + rank, dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    per_step = None
    for i in range(args.warmup):
        l0 = kernel_launches()
        net.step(x, y, SIGMA_V)
        if i == 1:
            per_step = kernel_launches() - l0  # the captured (or eager) step's launches
    torch.cuda.synchronize()

    L = lib()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    launches0 = kernel_launches()
    with ClockSampler(dev.index if dev.index is not None else 0) as clocks:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            net.step(x, y, SIGMA_V)
            ends[i].record()
        torch.cuda.synchronize()
        barrier()
    launches = kernel_launches() - launches0
    if graphed:
        # replays launch without passing through the library's host calls
        launches = per_step * args.steps
    step_s = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) * 1e-3
    # Per-entry timing after the timed region (the timed steps carry no events
    # of their own): CUDA events around every library call. One GPU with a
    # captured step: the step is captured once more with the events as graph
    # nodes and replayed, so each interval holds the call's kernels without the
    # host's launch gaps. Otherwise eager steps (host gaps included).
    fam_steps = min(3, args.steps)
    dp_timer = CollectiveTimer() if world > 1 else None
    captured = graphed and world == 1
    timer = LaunchTimer(external=captured)
    if captured:
        timed_graph = net._graph
        net._graph = (timed_graph[0], None, None, None, None)  # capture again, hook on
        for i in range(fam_steps):
            flush.zero_()
            L.hook = timer if i == 0 else None
            net.step(x, y, SIGMA_V)
            L.hook = None
            torch.cuda.synchronize()
            timer.harvest()
        net._graph = timed_graph
    else:
        net.cuda_graph = False
        for _ in range(fam_steps):
            flush.zero_()
            L.hook = timer
            if dp_timer is not None:
                net.reducer.timer = dp_timer
            net.step(x, y, SIGMA_V)
            L.hook = None
            if dp_timer is not None:
                net.reducer.timer = None
        net.cuda_graph = graphed
    torch.cuda.synchronize()
    barrier()
    fam, other = timer.summary()
    dp_times = dp_timer.summary(fam_steps) if dp_timer is not None else None

    # end to end through the public API: pinned host inputs in, predictions out
    xh, yh = x.cpu().pin_memory(), y.cpu().pin_memory()
    xd, yd = torch.empty_like(x), torch.empty_like(y)
    mu_h = torch.empty(y.shape, pin_memory=True)
    var_h = torch.empty(y.shape, pin_memory=True)
    e_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.zero_()
        e_starts[i].record()
        xd.copy_(xh, non_blocking=True)
        yd.copy_(yh, non_blocking=True)
        mu, var = net.step(xd, yd, SIGMA_V)
        mu_h.copy_(mu, non_blocking=True)
        var_h.copy_(var, non_blocking=True)
        e_ends[i].record()
    torch.cuda.synchronize()
    barrier()
    e2e_s = sum(s.elapsed_time(e) for s, e in zip(e_starts, e_ends)) * 1e-3

    # error word of the tensor-core kernels: a bounded wait that ran out inside
    # the timed or end-to-end steps would have left outputs incomplete
    status = device_status(reset=True)
    replicas = replica_check(net, dev, world) if world > 1 else None

    if world > 1:
        t = torch.tensor([step_s, e2e_s, float(status != 0)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_s, e2e_s, bad = t.tolist()
        status = status or int(bad)

    # North-star sub-records from the same run: the MLP step at the same number
    # of GPUs, and (one GPU) the Linear sweep's 8192 x 4096 x 4096 headline shape.
    tf32 = tf32_peak_tflops(dev) if rank == 0 or world == 1 else None
    sub = {}
    if not args.no_subrecords:
        if args.workload != "mlp":
            sub["mlp"] = mlp_subrecord(dev, rank, world, args.steps, args.warmup, flush, barrier,
                                       args.dp_graph)
        if world == 1:
            row = sweep_rows([(8192, 4096)], dev, 5, 3, tf32)[0]
            sub["sweep_8192x4096"] = {k: row[k] for k in ("forward", "backward", "update")}
            sub["sweep_8192x4096"]["peak_3xtf32_tflops"] = tf32 / 3.0
    status = status or device_status(reset=True)

    peaks = measured_peaks()
    if rank != 0:
        return
    value = args.steps * B * world / step_s
    dom_name, dom = max(fam.items(), key=lambda kv: kv[1]["seconds"]) if fam else (None, None)
    peak3 = tf32 / 3.0 if tf32 else None
    roof = None
    if dom is not None:
        achieved = dom["flops"] / dom["seconds"] / 1e12
        roof = {"bound": "tensor", "kernel": dom_name, "achieved": achieved, "peak": peak3,
                "unit": "TFLOP/s", "frac": achieved / peak3 if peak3 else None,
                "traffic": MEASURED_TRAFFIC.get((args.workload, dom_name)),
                "traffic_unit": "bytes per launch (ncu)",
                "peak_source": f"measured cuBLAS TF32 burst {tf32:.0f} TF/s / 3 (3xTF32-effective)",
                "launches": dom["launches"],
                "share_of_step": dom["seconds"] / fam_steps / (step_s / args.steps)}
    line = {
        "metric": WORKLOADS[args.workload]["metric"], "value": value, "unit": "samples/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * step_s / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "batch_per_gpu": B, "global_batch": B * world,
                   "sigma_v": SIGMA_V, "parallelism": f"dp{world}",
                   "l2": "flushed between steps (256 MiB write outside the timed events)",
                   "cuda_graph": graphed},
        "e2e": {"value": args.steps * B * world / e2e_s, "unit": "samples/s",
                "h2d_bytes_per_step": (xh.numel() + yh.numel()) * 4,
                "d2h_bytes_per_step": (mu_h.numel() + var_h.numel()) * 4},
        "gpu_launches": int(launches),
        "roofline": roof,
        "entry_timing": ("events as nodes of a captured step, replayed" if captured
                         else "events around eager calls (host launch gaps included)"),
        "kernels": {k: {"launches": v["launches"], "ms_per_step": 1e3 * v["seconds"] / fam_steps,
                        "tflops": v["flops"] / v["seconds"] / 1e12} for k, v in fam.items()},
        # every other library entry of the step (CUDA events around each call);
        # gbs = algorithmic bytes / time, hbm_frac against the measured copy bandwidth
        "entries": {k: {"launches": v["launches"], "ms_per_step": 1e3 * v["seconds"] / fam_steps,
                        **({"gbs": v["bytes"] / v["seconds"] / 1e9,
                            "hbm_frac": (v["bytes"] / v["seconds"] / 1e9 / peaks["hbm_gbs"]
                                         if peaks.get("hbm_gbs") else None)}
                           if v["bytes_known"] and v["bytes"] > 0 else {})}
                    for k, v in sorted(other.items(), key=lambda kv: -kv[1]["seconds"])},
        "clocks": clocks.summary(),
        "peaks": {"tf32_cublas_tflops": tf32, "tf32_source": "cuBLAS 8192^3, median of 9",
                  "hbm_gbs": peaks.get("hbm_gbs"), "bf16_tflops": peaks.get("bf16_tflops")},
        "device_status": status,
        **({"replicas_bit_identical": replicas} if replicas is not None else {}),
        # data-parallel collectives on the compute stream (CUDA events, rank 0,
        # eager steps after the timed ones): SyncBN statistics all-reduces, the
        # waits for the gradient buckets at the end of the backward (the part of
        # their all-reduces not hidden behind the backward), the update from the
        # reduced sums
        **({"dp_collectives": dp_times} if dp_times is not None else {}),
        **({"subrecords": sub} if sub else {}),
    }
    if world == 1 and not args.no_cpu_baseline:
        r = cpu_rate(args.workload, steps=5, warmup=1, budget_s=30.0)
        line["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)
    if status != 0:
        raise RuntimeError(f"a tensor-core kernel wait ran out during the run (code {status}); "
                           "the numbers above are not valid")


def replica_check(net, dev, world: int) -> bool:
    """True if every rank holds bit-identical parameters (an integer checksum of
    every parameter's bits, gathered from all ranks)."""
    acc = torch.zeros(2, dtype=torch.int64, device=dev)
    for leaf in net.leaves():
        for name in ("mw", "Sw", "mb", "Sb", "running_mean", "running_var"):
            t = getattr(leaf, name, None)
            if t is not None:
                bits = t.detach().contiguous().view(torch.int32).reshape(-1).to(torch.int64)
                acc[0] += bits.sum()
                acc[1] += (bits * torch.arange(1, bits.numel() + 1, device=dev) % 1000003).sum()
    allv = [torch.empty_like(acc) for _ in range(world)]
    dist.all_gather(allv, acc)
    return all(torch.equal(v, allv[0]) for v in allv)


def mlp_subrecord(dev, rank: int, world: int, steps: int, warmup: int, flush, barrier,
                  dp_graph: bool = False) -> dict:
    """MLP 784-256-128-10 Sequential.step, batch 256 per GPU, at the run's number
    of GPUs (data parallel for N > 1), timed like the main workload."""
    import triton_tagi as TT

    B = WORKLOADS["mlp"]["batch"]
    torch.manual_seed(4321)
    graphed = world == 1 or dp_graph
    net = TT.Sequential(build_layers("mlp", TT, dev), device=dev, cuda_graph=graphed)
    _NETS.append(net)
    if world > 1:
        from triton_tagi.distributed import DataParallel

        DataParallel(net, capturable=dp_graph)
    x, y = make_batch("mlp", B, 300 + rank, dev)
    for _ in range(max(3, warmup)):
        net.step(x, y, SIGMA_V)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        flush.zero_()
        starts[i].record()
        net.step(x, y, SIGMA_V)
        ends[i].record()
    torch.cuda.synchronize()
    barrier()
    t = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) * 1e-3
    if world > 1:
        tt = torch.tensor([t], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = tt.item()
    return {"metric": WORKLOADS["mlp"]["metric"], "value": steps * B * world / t,
            "unit": "samples/s", "ms_per_step": 1e3 * t / steps, "batch_per_gpu": B,
            "global_batch": B * world, "steps": steps, "cuda_graph": graphed,
            "l2": "flushed between steps"}


def sweep_rows(shapes, dev, steps: int, warmup: int, peak_tf32: float) -> list[dict]:
    """Linear op sweep rows: forward (mean+var), backward delta and weight sums
    with the capped update of each (M, K = N) shape, each launch timed with CUDA
    events (L2 flushed before every launch), median over ``steps``."""
    import triton_tagi as TT
    from triton_tagi._lib import lib, stream
    from triton_tagi.layers._params import weight_param_backward

    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)
    L = lib()
    rows = []
    for M, K in shapes:
        N = K
        g = torch.Generator(device=dev).manual_seed(M + K)
        ma = torch.randn(M, K, device=dev, generator=g)
        Sa = torch.rand(M, K, device=dev, generator=g) * (1e-2 - 1e-4) + 1e-4
        lin = TT.Linear(K, N, device=dev)
        lin.mw = torch.randn(K, N, device=dev, generator=g) / K**0.5
        lin.Sw = (torch.rand(K, N, device=dev, generator=g) + 0.5) / K
        lin.mb = torch.zeros(1, N, device=dev)
        lin.Sb = torch.full((1, N), 1e-3, device=dev)
        dmz = torch.randn(M, N, device=dev, generator=g) * 0.1
        dSz = -torch.rand(M, N, device=dev, generator=g) * 1e-2
        d_ma = torch.empty(M, K, device=dev)
        d_Sa = torch.empty(M, K, device=dev)
        ws_n = L.size("tagi_store_workspace_size", M, K, N)
        ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)

        def fwd():
            lin.forward(ma, Sa)

        def bwd():
            L("tagi_linear_backward_delta", dmz.data_ptr(), dSz.data_ptr(), lin.mw.data_ptr(),
              d_ma.data_ptr(), d_Sa.data_ptr(), M, K, N, ws.data_ptr() if ws_n else None,
              ws_n, stream(dmz))

        def upd():
            lin._set_param_mode("update", 3.0)
            weight_param_backward(lin, ma, K, (dmz, dSz), (0, 0, N, 1), M, K, N, True)
            lin._set_param_mode("deltas")

        row = {"M": M, "K": K, "N": N}
        for name, fn, flops in (("forward", fwd, 6.0 * M * N * K),
                                ("backward", bwd, 4.0 * M * N * K),
                                ("update", upd, 4.0 * M * N * K)):
            for _ in range(warmup):
                fn()
            times = []
            for _ in range(steps):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn()
                b.record()
                b.synchronize()
                times.append(a.elapsed_time(b) * 1e-3)
            t = statistics.median(times)
            row[name] = {"ms": 1e3 * t, "tflops": flops / t / 1e12,
                         "frac": flops / t / 1e12 / (peak_tf32 / 3.0),
                         "samples_per_s": M / t}
        rows.append(row)
        del ma, Sa, lin, dmz, dSz, d_ma, d_Sa, ws
    return rows


def sweep_arm(args, rank: int, world: int, local: int) -> None:
    """Linear op sweep, every shape."""
    from triton_tagi._lib import kernel_launches

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shapes = [tuple(int(v) for v in args.shape.split(","))] if args.shape else SWEEP
    peak_tf32 = tf32_peak_tflops(dev)
    launches0 = kernel_launches()
    with ClockSampler(dev.index or 0) as clocks:
        rows = sweep_rows(shapes, dev, args.steps, args.warmup, peak_tf32)
    if rank != 0:
        return
    top = max(rows, key=lambda r: r["M"] * r["K"])
    step_s = sum(top[n]["ms"] for n in ("forward", "backward", "update")) * 1e-3
    fwd = top["forward"]
    line = {
        "metric": WORKLOADS["swp"]["metric"], "value": fwd["tflops"], "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * step_s,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "swp", "shapes": [[r["M"], r["K"]] for r in rows],
                   "l2": "flushed before every timed launch (256 MiB write)"},
        "roofline": {"bound": "tensor", "kernel": "moment_forward", "achieved": fwd["tflops"],
                     "peak": peak_tf32 / 3.0, "unit": "TFLOP/s", "frac": fwd["frac"],
                     "traffic": MEASURED_TRAFFIC.get(("swp", "moment_forward"))
                     if (top["M"], top["K"]) == (8192, 4096) else None,
                     "traffic_unit": "bytes per launch (ncu)",
                     "peak_source": f"measured cuBLAS TF32 burst {peak_tf32:.0f} TF/s "
                                    "(median of 9) / 3"},
        "sweep": rows, "gpu_launches": int(kernel_launches() - launches0),
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


MICRO = ("remax", "col2im", "im2col", "bn")


def micro_arm(which: str) -> None:
    """Profiling drivers: one library entry on the benchmark shapes, 3 warm-up
    and 10 timed calls per shape (CUDA events), one line per shape. remax: the
    transformer's score rows (32768 x 512, a quarter of one layer's);
    col2im / im2col: the ResNet-18 (batch 128) stride-2 gathers and the patches
    of the weight sums; bn: the BatchNorm training forward (with and without the
    residual stream) and backward on the four ResNet-18 stage shapes."""
    import triton_tagi  # noqa: F401  (loads the library)
    from triton_tagi._lib import lib
    from triton_tagi.layers.remax import triton_remax

    L = lib()
    st = torch.cuda.current_stream().cuda_stream

    def timed(fn, n=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return 1e3 * e0.elapsed_time(e1) / n

    g = torch.Generator(device="cuda").manual_seed(0)
    N = 128
    if which == "bn":
        # training forward (with and without the residual stream) and backward
        # (ReLU Jacobian, delta sums, capped update) on the four stage shapes
        for C, H in ((64, 32), (128, 16), (256, 8), (512, 4)):
            mz = torch.randn(N, C, H, H, device="cuda", generator=g)
            Sz = torch.rand(N, C, H, H, device="cuda", generator=g) + 0.1
            rm, rS = torch.randn_like(mz), torch.rand_like(Sz)
            prm = [torch.rand(C, device="cuda", generator=g) + 0.5 for _ in range(8)]
            mean, var, rmean, rvar, mg, Sg, mb, Sb = prm
            ma, Sa, mh = torch.empty_like(mz), torch.empty_like(mz), torch.empty_like(mz)
            outs = [torch.empty_like(mz) for _ in range(2)]
            grads = torch.empty(4 * C, device="cuda", dtype=torch.float64)
            dsums = torch.empty(2 * C, device="cuda", dtype=torch.float64)
            n = mz.numel()
            for add in (False, True):
                us = timed(lambda: L("tagi_bn_train_forward", mz.data_ptr(), Sz.data_ptr(),
                                     mean.data_ptr(), var.data_ptr(), rmean.data_ptr(),
                                     rvar.data_ptr(), mg.data_ptr(), Sg.data_ptr(), mb.data_ptr(),
                                     Sb.data_ptr(), ma.data_ptr(), Sa.data_ptr(), mh.data_ptr(),
                                     rm.data_ptr() if add else None,
                                     rS.data_ptr() if add else None, N, C, H * H, 0, 0, 0.1,
                                     1e-5, st))
                nbytes = (28 if add else 20) * n
                print(f"bn_train_forward C{C} H{H}{' +add' if add else ''}: {us:.1f} us, "
                      f"{nbytes / us / 1e3:.0f} GB/s")
            us = timed(lambda: L("tagi_bn_backward", ma.data_ptr(), Sa.data_ptr(), mh.data_ptr(),
                                 var.data_ptr(), mg.data_ptr(), outs[0].data_ptr(),
                                 outs[1].data_ptr(), rS.data_ptr(), grads.data_ptr(),
                                 dsums.data_ptr(), N, C, H * H, 1e-5, Sg.data_ptr(),
                                 mb.data_ptr(), Sb.data_ptr(), 2.0, st))
            print(f"bn_backward C{C} H{H}: {us:.1f} us, {24 * n / us / 1e3:.0f} GB/s")
        return
    if which == "remax":
        mz = torch.randn(32768, 512, device="cuda", generator=g) * 2
        Sz = torch.rand(32768, 512, device="cuda", generator=g) * 2 + 1e-3
        us = timed(lambda: triton_remax(mz, Sz))
        print(f"remax 32768x512: {us:.1f} us, {20 * mz.numel() / us / 1e3:.0f} GB/s")
        return
    shapes = {"col2im": ((64, 32, 3, 1, 2), (128, 16, 3, 1, 2), (256, 8, 3, 1, 2),
                         (64, 32, 2, 0, 1), (128, 16, 2, 0, 1), (256, 8, 2, 0, 1)),
              "im2col": ((64, 32, 3, 1, 2), (128, 16, 3, 1, 1), (128, 16, 3, 1, 2),
                         (256, 8, 3, 1, 1), (256, 8, 3, 1, 2), (512, 4, 3, 1, 1),
                         (64, 32, 2, 0, 1))}[which]
    for C, H, k, p, pt in shapes:
        s = 2 if (which == "col2im" or pt == 2 or k == 2) else 1
        Ho = (H + (p if pt == 2 else 2 * p) - k) // s + 1
        K = C * k * k
        if which == "col2im":
            cm = torch.randn(N * Ho * Ho, K, device="cuda", generator=g)
            cS = torch.rand(N * Ho * Ho, K, device="cuda", generator=g)
            dm = torch.empty(N, C, H, H, device="cuda")
            dS = torch.empty_like(dm)
            us = timed(lambda: L("tagi_col2im", cm.data_ptr(), cS.data_ptr(), dm.data_ptr(),
                                 dS.data_ptr(), N, C, H, H, k, s, p, pt, 0, st))
            nbytes = 8 * (cm.numel() + dm.numel())
        else:
            x = torch.randn(N, C, H, H, device="cuda", generator=g)
            pm = torch.empty(N * Ho * Ho, K, device="cuda")
            us = timed(lambda: L("tagi_im2col", x.data_ptr(), None, pm.data_ptr(), None, N, C,
                                 H, H, k, s, p, pt, st))
            nbytes = 4 * (x.numel() + pm.numel())
        print(f"{which} C{C} H{H} k{k} s{s}: {us:.1f} us, {nbytes / us / 1e3:.0f} GB/s")


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="r18")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="mlp/cnn: run the steps eagerly instead of replaying a CUDA graph")
    ap.add_argument("--shape", default=None, help="swp workload: one 'M,K' shape (K = N)")
    ap.add_argument("--batch", type=int, default=None,
                    help="per-GPU batch (default: the workload's configuration; smaller "
                         "batches are for profiling captures only)")
    ap.add_argument("--no-dp-graph", dest="dp_graph", action="store_false",
                    help="N > 1: run the data-parallel step eagerly instead of replaying it "
                         "(NCCL collectives included) from a CUDA graph")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="skip the MLP and sweep sub-records of the default line")
    ap.add_argument("--micro", choices=MICRO, default=None,
                    help="profiling driver: time one library entry on the benchmark shapes "
                         "instead of a workload step (no JSON line)")
    args = ap.parse_args()
    if args.micro is not None:
        micro_arm(args.micro)
        return
    if args.batch is not None:
        WORKLOADS[args.workload] = dict(WORKLOADS[args.workload], batch=args.batch)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)  # rank 0 only; no process group needed
        return
    if args.workload == "swp":
        sweep_arm(args, rank, world, local)
        return
    if world > 1:
        import datetime

        # NCCL's gradient all-reduces run beside the backward contractions; with
        # at most 8 channels they take fewer SMs from them (measured at two GPUs:
        # 13.37 -> 13.18 ms per ResNet-18 step) and still finish inside the backward
        os.environ.setdefault("NCCL_MAX_NCHANNELS", "8")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        our_arm(args, rank, world, local)
    finally:
        # graphs that hold NCCL calls go before the process group does
        for n in _NETS:
            n.release_graph()
        for n in _NETS:  # peer exchange buffers (collective, same order on every rank)
            if getattr(n, "reducer", None) is not None:
                n.reducer.close()
        _NETS.clear()
        import gc

        gc.collect()
        torch.cuda.synchronize()
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
