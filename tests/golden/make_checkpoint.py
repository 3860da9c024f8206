"""Write a checkpoint with the reference implementation's own RunDir, for the
format-compatibility test (tests/test_checkpoint.py).

Run in a container where the triton-tagi sources are available (read-only):

    python tests/golden/make_checkpoint.py /path/to/triton-tagi

Builds a small network with the reference's layer classes on the CPU (an MLP
head after a ResBlock with a projection and a BatchNorm2D), sets every saved
tensor to seeded values, saves it with ``RunDir.save_checkpoint`` and copies
the file to ``tests/golden/ref_checkpoint.pt``. The GPU box never runs this.
"""

from __future__ import annotations

import os
import shutil
import sys
import tempfile
from pathlib import Path

OUT = Path(__file__).resolve().parent


def topology(L, device="cpu"):
    """The layer list both implementations build for the test."""
    return [L.Conv2D(3, 4, 3, padding=1, device=device), L.ReLU(),
            L.BatchNorm2D(4, device=device),
            L.ResBlock(4, 8, 2, device=device),
            L.AvgPool2D(2), L.Flatten(), L.Linear(8 * 2 * 2, 5, device=device), L.Remax()]


def main(ref_root: str) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch
    import triton_tagi as R

    torch.manual_seed(0)
    net = R.Sequential(topology(R), device="cpu")
    g = torch.Generator().manual_seed(1)
    for layer in net.layers:
        for sub in getattr(layer, "_learnable", [layer]):
            for a in ("mw", "Sw", "mb", "Sb", "running_mean", "running_var"):
                t = getattr(sub, a, None)
                if isinstance(t, torch.Tensor):
                    t.data.copy_(torch.rand(t.shape, generator=g) + 0.1)
    with tempfile.TemporaryDirectory() as d:
        run = R.RunDir("synthetic", "small", "tagi", base=d)
        path = run.save_checkpoint(net, 7, {"note": "format test", "width": 4})
        shutil.copy(path, OUT / "ref_checkpoint.pt")


if __name__ == "__main__":
    main(sys.argv[1])
