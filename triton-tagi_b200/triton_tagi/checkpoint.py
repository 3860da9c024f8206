"""Run directories, checkpoints and metrics logs (drop-in for
triton_tagi/checkpoint.py).

A run writes everything under ``{base}/{dataset}_{arch}_{optimizer}_{stamp}/``:
``config.json``, ``metrics.csv``, ``checkpoints/epoch_NNNN.pt`` and ``figures/``
(checkpoint.py:30-56). The checkpoint file is the reference's, so models move
between the two implementations in both directions (checkpoint.py:63-77,
165-214): a ``torch.save`` of

    {"epoch": int, "config": dict,
     "net_state": {index in net.layers: {attr: CPU tensor}
                                        | [one such dict per sub-layer]}}

where ``attr`` runs over ``mw, Sw, mb, Sb, running_mean, running_var`` (those
the layer has) and containers with sub-layers (``ResBlock``) store a list in
their ``_learnable`` order (conv1, bn1, conv2, bn2[, proj_conv, proj_bn]).
Loading copies into the existing parameter tensors, on the network's device.
"""

from __future__ import annotations

import csv
import json
from datetime import datetime
from pathlib import Path
from typing import Any, Callable

import torch

from .base import LearnableLayer
from .network import Sequential

STATE_ATTRS = ("mw", "Sw", "mb", "Sb", "running_mean", "running_var")


def layer_state(layer) -> dict[str, torch.Tensor]:
    """The saved tensors of one leaf layer (copies on the CPU)."""
    return {a: getattr(layer, a).detach().cpu().clone() for a in STATE_ATTRS
            if getattr(layer, a, None) is not None}


def net_state(net: Sequential) -> dict[int, Any]:
    """``net_state`` of a checkpoint: learnable layers by their index."""
    out: dict[int, Any] = {}
    for i, layer in enumerate(net.layers):
        subs = getattr(layer, "_learnable", None)
        if subs is not None:
            states = [layer_state(s) for s in subs]
            if any(states):
                out[i] = states
        elif isinstance(layer, LearnableLayer):
            st = layer_state(layer)
            if st:
                out[i] = st
    return out


def _copy_into(layer, saved: dict[str, torch.Tensor], device: torch.device) -> None:
    for a in STATE_ATTRS:
        if a in saved and getattr(layer, a, None) is not None:
            getattr(layer, a).data.copy_(saved[a].to(device))


def restore_net_state(net: Sequential, state: dict[int, Any]) -> None:
    """Copy a checkpoint's ``net_state`` into ``net``'s parameter tensors."""
    for i, layer in enumerate(net.layers):
        saved = state.get(i)
        if saved is None:
            continue
        if isinstance(saved, list):
            for sub, sub_saved in zip(layer._learnable, saved):
                _copy_into(sub, sub_saved, net.device)
        else:
            _copy_into(layer, saved, net.device)


class RunDir:
    """The directory of one training run (checkpoint.py:30-114)."""

    def __init__(self, dataset: str, arch: str, optimizer: str, base: str = "runs") -> None:
        stamp = datetime.now().strftime("%Y%m%d-%H%M%S")
        self.path = Path(base) / f"{dataset}_{arch}_{optimizer}_{stamp}"
        self.checkpoints = self.path / "checkpoints"
        self.figures = self.path / "figures"
        self.config_json = self.path / "config.json"
        self.metrics_csv = self.path / "metrics.csv"
        self.path.mkdir(parents=True, exist_ok=True)
        self.checkpoints.mkdir()
        self.figures.mkdir()

    def save_config(self, config: dict[str, Any]) -> None:
        self.config_json.write_text(json.dumps(config, indent=2))

    def save_checkpoint(self, net: Sequential, epoch: int, config: dict[str, Any]) -> Path:
        """Writes ``checkpoints/epoch_{epoch:04d}.pt`` and returns its path."""
        path = self.checkpoints / f"epoch_{epoch:04d}.pt"
        torch.save({"epoch": epoch, "config": config, "net_state": net_state(net)}, path)
        return path

    def load_checkpoint(self, net: Sequential, path: str | Path | None = None) -> int:
        """Restores ``net`` from ``path`` (default: the last ``epoch_*.pt``) and
        returns the saved epoch."""
        if path is None:
            found = sorted(self.checkpoints.glob("epoch_*.pt"))
            if not found:
                raise FileNotFoundError(f"No checkpoints found in {self.checkpoints}")
            path = found[-1]
        ck = torch.load(path, map_location=net.device, weights_only=False)
        restore_net_state(net, ck["net_state"])
        return ck["epoch"]

    def append_metrics(self, epoch: int, **metrics: float) -> None:
        """Appends one row to ``metrics.csv`` (header from the first row's keys;
        floats written with 6 significant digits)."""
        row = {"epoch": epoch, **metrics}
        new = not self.metrics_csv.exists()
        with open(self.metrics_csv, "a", newline="") as f:
            w = csv.DictWriter(f, fieldnames=list(row))
            if new:
                w.writeheader()
            w.writerow({k: (f"{v:.6g}" if isinstance(v, float) else v) for k, v in row.items()})

    def __repr__(self) -> str:
        return f"RunDir({self.path})"


def load_model(path: str | Path, build: Callable[[dict[str, Any]], Sequential],
               device: str | torch.device = "cuda") -> tuple[Sequential, dict[str, Any], int]:
    """(net, config, epoch): ``build(config)`` makes the topology, then the saved
    parameters are copied in (checkpoint.py:117-162)."""
    device = torch.device(device)
    ck = torch.load(path, map_location=device, weights_only=False)
    net = build(ck["config"])
    if hasattr(net, "to"):
        net = net.to(device)
    restore_net_state(net, ck["net_state"])
    return net, ck["config"], ck["epoch"]
