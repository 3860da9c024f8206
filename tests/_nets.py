"""Network builders shared by the parity tests.

``build(name, L)`` assembles one of the golden-trajectory topologies from a
namespace ``L`` that provides the triton-tagi layer classes (the CPU oracle's
or this library's); ``params(layers)`` lists learnable tensors in the order
``tests/golden/make_golden.py`` stored them, and ``load(layers, arrays)``
overwrites them in place of the random initialisation.
"""

from __future__ import annotations

import numpy as np
import torch


def build(name: str, L, device="cpu"):
    d = dict(device=device)
    if name == "mlp":
        return [L.Linear(784, 64, **d), L.ReLU(), L.Linear(64, 32, **d), L.ReLU(),
                L.Linear(32, 10, **d), L.Remax()]
    if name == "cnn":
        return [L.Conv2D(3, 8, 5, padding=2, **d), L.ReLU(), L.AvgPool2D(2),
                L.Conv2D(8, 16, 5, padding=2, **d), L.BatchNorm2D(16, **d), L.ReLU(),
                L.AvgPool2D(2), L.Flatten(), L.Linear(16 * 4 * 4, 32, **d), L.ReLU(),
                L.Linear(32, 10, **d), L.Remax()]
    if name == "res":
        kw = dict(gain_w=0.1, gain_b=0.1, **d)
        return [L.Conv2D(3, 8, 3, stride=1, padding=1, **kw), L.ReLU(), L.BatchNorm2D(8, **kw),
                L.ResBlock(8, 8, stride=1, **kw), L.ResBlock(8, 16, stride=2, **kw),
                L.AvgPool2D(4), L.Flatten(), L.Linear(16, 10, **kw), L.Remax()]
    if name == "tfm":
        V, E, H, S = 16, 32, 4, 8
        return [L.Embedding(V, E, input_size=S, scale=0.25, **d), L.PositionalEncoding(E, **d),
                L.MultiheadAttentionV2(E, H, S, bias=False, **d), L.RMSNorm(E, **d),
                L.Linear(E, 64, **d), L.ReLU(), L.Linear(64, E, **d), L.Linear(E, V, **d)]
    raise KeyError(name)


def _leaves(layers):
    out = []
    for layer in layers:
        if hasattr(layer, "_learnable"):
            out += list(layer._learnable)
        elif hasattr(layer, "q_proj"):
            out += [layer.q_proj, layer.k_proj, layer.v_proj]
        elif getattr(layer, "mw", None) is not None:
            out.append(layer)
    return out


def _names(layer):
    names = [n for n in ("mw", "Sw", "mb", "Sb") if getattr(layer, n, None) is not None]
    if hasattr(layer, "running_mean"):
        names += ["running_mean", "running_var"]
    return names


def params(layers):
    return [getattr(leaf, n) for leaf in _leaves(layers) for n in _names(leaf)]


def load(layers, arrays, device="cpu", dtype=torch.float32):
    """Assign golden arrays to the layers' tensors (same order as ``params``)."""
    i = 0
    for leaf in _leaves(layers):
        for n in _names(leaf):
            cur = getattr(leaf, n)
            new = torch.as_tensor(np.asarray(arrays[i]), dtype=dtype, device=device)
            assert tuple(new.shape) == tuple(cur.shape), (n, new.shape, cur.shape)
            setattr(leaf, n, new.contiguous())
            i += 1
    assert i == len(arrays)


def golden_params(z, step: int):
    keys = sorted(k for k in z.files if k.startswith(f"p{step}_"))
    return [z[k] for k in keys]


def build_config(name: str, L, device="cpu", width: float = 1.0):
    """The benchmark configurations (MLP, CNN, ResNet-18, transformer);
    ``width`` scales channels for CPU-affordable parity runs."""
    d = dict(device=device)
    if name == "mlp":
        return [L.Linear(784, 256, **d), L.ReLU(), L.Linear(256, 128, **d), L.ReLU(),
                L.Linear(128, 10, **d), L.Remax()]
    if name == "cnn":
        return [L.Conv2D(3, 32, 5, padding=2, **d), L.ReLU(), L.AvgPool2D(2),
                L.Conv2D(32, 64, 5, padding=2, **d), L.BatchNorm2D(64, **d), L.ReLU(),
                L.AvgPool2D(2),
                L.Conv2D(64, 64, 5, padding=2, **d), L.ReLU(), L.AvgPool2D(2),
                L.Flatten(), L.Linear(1024, 256, **d), L.ReLU(), L.Linear(256, 10, **d),
                L.Remax()]
    if name == "r18":
        c = [max(1, int(round(64 * width * m))) for m in (1, 2, 4, 8)]
        kw = dict(gain_w=0.1, gain_b=0.1, **d)
        return [L.Conv2D(3, c[0], 3, stride=1, padding=1, **kw), L.ReLU(),
                L.BatchNorm2D(c[0], **kw),
                L.ResBlock(c[0], c[0], stride=1, **kw), L.ResBlock(c[0], c[0], stride=1, **kw),
                L.ResBlock(c[0], c[1], stride=2, **kw), L.ResBlock(c[1], c[1], stride=1, **kw),
                L.ResBlock(c[1], c[2], stride=2, **kw), L.ResBlock(c[2], c[2], stride=1, **kw),
                L.ResBlock(c[2], c[3], stride=2, **kw), L.ResBlock(c[3], c[3], stride=1, **kw),
                L.AvgPool2D(4), L.Flatten(), L.Linear(c[3], 10, **kw), L.Remax()]
    if name == "tfm":
        V, E, H, S, blocks = 64, int(512 * width), 8, 512, 4
        layers = [L.Embedding(V, E, input_size=S, scale=0.25, **d), L.PositionalEncoding(E, **d)]
        for _ in range(blocks):
            layers += [L.MultiheadAttentionV2(E, H, S, bias=False, **d), L.RMSNorm(E, **d),
                       L.Linear(E, 4 * E, **d), L.ReLU(), L.Linear(4 * E, E, **d)]
        return layers + [L.Linear(E, V, **d)]
    raise KeyError(name)


def copy_params(src_layers, dst_layers, device) -> None:
    """Copy every learnable tensor (and BN running stats) from one net to another."""
    load(dst_layers, [t.detach().cpu().numpy() for t in params(src_layers)], device=device)


def sync_bn_state(src_layers, dst_layers) -> None:
    """Carry BatchNorm's first-call flag across (the oracle calls it ``_init``)."""
    def bns(layers):
        return [l for l in _leaves(layers) if hasattr(l, "running_mean")]
    for a, b in zip(bns(src_layers), bns(dst_layers)):
        flag = getattr(a, "_init", getattr(a, "_is_initialized", False))
        if hasattr(b, "_is_initialized"):
            b._is_initialized = flag
        else:
            b._init = flag
