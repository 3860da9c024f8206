"""Sequential container (drop-in for triton_tagi/network.py).

``step(x, y, σ_v)`` runs forward → innovation → backward → capped update and
returns the pre-update predictions, exactly as the reference
(network.py:119-152). Two differences in *how*, not *what*:

* With ``fuse_update=True`` (default) each learnable layer applies its capped
  update inside its backward, right after propagating the deltas with the
  pre-update weights; the weight-gradient kernel then writes the parameters
  directly and no delta tensors are allocated. Every layer's update only
  touches its own parameters, so the result is the reference's
  backward-then-update. ``fuse_update=False`` keeps the reference's call
  structure (``delta_*`` tensors stored, ``update`` applied afterwards).
* Under data parallelism (``triton_tagi.distributed``) the batch sums of every
  layer are all-reduced before the update and the cap factor uses the global
  batch, so every replica applies the single-batch closed form.

``cuda_graph=True`` replays each step from a CUDA graph: the first step with a
new input shape (or σ_v) runs eagerly, the next one is captured on static input
buffers and replayed, and later steps copy their inputs in and replay. A step
of small layers is a few dozen short kernels, so launch overhead otherwise
dominates it. The replayed kernels are the eager step's; returned predictions
are copies. Under data parallelism the step is captured only if the reducer
says its collectives can be (``DataParallel(capturable=True)``, NCCL): the
graph then holds the SyncBN and gradient all-reduces too, every rank replays
the same graph, and the capture is thread-local so that the communicator's
watchdog thread may keep polling; otherwise the step runs eagerly. The
captured graph is keyed on the input shapes, σ_v, ``fuse_update`` and every
layer's training flag, so ``train()`` / ``eval()`` lead to a new capture.

``check_device=True`` (or the environment variable ``TAGI_B200_CHECK=1``) reads
the tensor-core kernels' error word after every step (this synchronises) and
raises ``RuntimeError`` if a bounded wait inside a kernel ran out, in which case
that kernel's outputs are incomplete.
"""

from __future__ import annotations

import os

import torch
from torch import Tensor

from ._chain import backward_chain, forward_chain
from ._lib import check_device_status
from .base import LearnableLayer
from .layers.multihead_attention import MultiheadAttentionV2
from .layers.resblock import ResBlock
from .update.observation import compute_innovation
from .update.parameters import get_cap_factor


class Sequential:
    def __init__(self, layers: list, device="cuda", fuse_update: bool = True,
                 cuda_graph: bool = False, check_device: bool | None = None) -> None:
        self.device = torch.device(device)
        self.layers = layers
        self.fuse_update = fuse_update
        self.cuda_graph = cuda_graph
        if check_device is None:
            check_device = os.environ.get("TAGI_B200_CHECK", "0") == "1"
        self.check_device = check_device
        self._graph = None  # (key, CUDAGraph or None, static x, static y, outputs)
        self.reducer = None  # set by triton_tagi.distributed.DataParallel
        for layer in self.layers:
            if isinstance(layer, ResBlock):
                layer.device = self.device
                for sub in layer._learnable:
                    self._move_layer_to_device(sub)
            elif isinstance(layer, LearnableLayer):
                self._move_layer_to_device(layer)
            if hasattr(layer, "running_mean"):
                layer.running_mean = layer.running_mean.to(self.device)
                layer.running_var = layer.running_var.to(self.device)

    def _move_layer_to_device(self, layer) -> None:
        if isinstance(layer, MultiheadAttentionV2):
            layer.device = self.device
            for sub in (layer.q_proj, layer.k_proj, layer.v_proj):
                self._move_layer_to_device(sub)
            return
        if getattr(layer, "mw", None) is None:
            return
        layer.device = self.device
        for name in ("mw", "Sw", "mb", "Sb", "running_mean", "running_var"):
            t = getattr(layer, name, None)
            if t is not None:
                setattr(layer, name, t.to(self.device))

    def learnable_layers(self) -> list[LearnableLayer]:
        return [layer for layer in self.layers if isinstance(layer, LearnableLayer)]

    def leaves(self) -> list[LearnableLayer]:
        """Learnable layers that own parameters, in network order."""
        out = []
        for layer in self.learnable_layers():
            out += layer._leaves()
        return out

    def forward(self, x: Tensor) -> tuple[Tensor, Tensor]:
        return forward_chain(self.layers, x, torch.zeros_like(x))

    def step(self, x_batch: Tensor, y_batch: Tensor, sigma_v: float) -> tuple[Tensor, Tensor]:
        red = self.reducer
        if self.cuda_graph and x_batch.is_cuda and (
                red is None or getattr(red, "capturable", False)):
            out = self._graph_step(x_batch, y_batch, sigma_v)
        else:
            out = self._step(x_batch, y_batch, sigma_v)
        if self.check_device:
            check_device_status()
        return out

    def _modes(self) -> tuple:
        """Training flags of every layer (and sub-layer), in network order."""
        flags = []

        def walk(layer):
            flags.append(getattr(layer, "training", None))
            for sub in getattr(layer, "_learnable", ()):
                if sub is not layer:
                    walk(sub)

        for layer in self.layers:
            walk(layer)
        return tuple(flags)

    def _graph_step(self, x_batch: Tensor, y_batch: Tensor, sigma_v: float) -> tuple[Tensor, Tensor]:
        key = (tuple(x_batch.shape), x_batch.dtype, tuple(y_batch.shape), y_batch.dtype,
               float(sigma_v), x_batch.device, self.fuse_update, self._modes())
        if self._graph is None or self._graph[0] != key:
            # first step of this shape: eager (it also leaves every layer in its
            # steady state, e.g. BatchNorm's running statistics initialised)
            self._graph = (key, None, None, None, None)
            return self._step(x_batch, y_batch, sigma_v)
        _, graph, sx, sy, out = self._graph
        if graph is None:
            sx, sy = x_batch.clone(), y_batch.clone()
            graph = torch.cuda.CUDAGraph()
            mode = "thread_local" if self.reducer is not None else "global"
            with torch.cuda.graph(graph, capture_error_mode=mode):
                out = self._step(sx, sy, sigma_v)
            self._graph = (key, graph, sx, sy, out)
        else:
            sx.copy_(x_batch)
            sy.copy_(y_batch)
        graph.replay()
        return out[0].clone(), out[1].clone()

    def _step(self, x_batch: Tensor, y_batch: Tensor, sigma_v: float) -> tuple[Tensor, Tensor]:
        red = self.reducer
        global_batch = x_batch.shape[0] * (red.world_size if red is not None else 1)
        y_pred_mu, y_pred_var = self.forward(x_batch)
        delta_mu, delta_var = compute_innovation(y_batch, y_pred_mu, y_pred_var, sigma_v)
        cap = get_cap_factor(global_batch)
        mode = "sums" if red is not None else ("update" if self.fuse_update else "deltas")
        learn = self.learnable_layers()
        for layer in learn:
            layer._set_param_mode(mode, cap, red)
        first = self.layers[0] if self.layers else None
        try:
            if red is not None:
                red.begin_step()
            if isinstance(first, LearnableLayer):
                first._skip_input_delta = True  # the input's deltas are not used
            delta_mu, delta_var = backward_chain(self.layers, delta_mu, delta_var)
            if red is not None:
                red.finish_step(cap)
            for layer in learn:
                layer.update(cap)
        finally:
            if isinstance(first, LearnableLayer):
                first._skip_input_delta = False
            for layer in learn:
                layer._set_param_mode("deltas")
        return y_pred_mu, y_pred_var

    def release_graph(self) -> None:
        """Drop the captured step (a graph that holds NCCL calls must be released
        before the process group is destroyed)."""
        self._graph = None

    def train(self) -> None:
        for layer in self.layers:
            if hasattr(layer, "training"):
                layer.train()
        self._graph = None

    def eval(self) -> None:
        for layer in self.layers:
            if hasattr(layer, "training"):
                layer.eval()
        self._graph = None

    def __repr__(self):
        lines = ["Sequential("] + [f"  ({i}): {layer}" for i, layer in enumerate(self.layers)]
        return "\n".join(lines + [")"])

    def num_parameters(self) -> int:
        return sum(layer.num_parameters for layer in self.learnable_layers())

    def get_attention_scores(self) -> dict[int, tuple[Tensor, Tensor]]:
        out = {i: layer.get_attention_scores() for i, layer in enumerate(self.layers)
               if isinstance(layer, MultiheadAttentionV2)}
        if not out:
            raise RuntimeError("No attention layers in this Sequential.")
        return out
