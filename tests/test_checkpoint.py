"""Checkpoint format compatibility with the reference (triton_tagi/checkpoint.py).

``tests/golden/ref_checkpoint.pt`` was written by the reference's own
``RunDir.save_checkpoint`` (``tests/golden/make_checkpoint.py``) for a network
with a Conv2D, a BatchNorm2D, a ResBlock with projection and a Linear head.
These tests need no GPU: parameters live on the CPU until a layer computes.
"""

from __future__ import annotations

import csv
import importlib.util
import json
from pathlib import Path

import torch

import triton_tagi as TT

GOLDEN = Path(__file__).resolve().parent / "golden"


def _topology():
    spec = importlib.util.spec_from_file_location("make_checkpoint", GOLDEN / "make_checkpoint.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.topology


def _build(cfg=None):
    torch.manual_seed(123)
    return TT.Sequential(_topology()(TT, "cpu"), device="cpu")


def _same_state(a, b):
    assert a.keys() == b.keys()
    for i in a:
        x, y = a[i], b[i]
        if isinstance(x, list):
            assert isinstance(y, list) and len(x) == len(y)
            pairs = zip(x, y)
        else:
            pairs = [(x, y)]
        for dx, dy in pairs:
            assert dx.keys() == dy.keys(), (i, dx.keys(), dy.keys())
            for k in dx:
                assert dx[k].dtype == dy[k].dtype and dx[k].shape == dy[k].shape, (i, k)
                assert torch.equal(dx[k], dy[k]), (i, k)


def test_reference_checkpoint_loads_into_this_implementation():
    ref = torch.load(GOLDEN / "ref_checkpoint.pt", weights_only=False)
    net, cfg, epoch = TT.load_model(GOLDEN / "ref_checkpoint.pt", _build, device="cpu")
    assert epoch == ref["epoch"] == 7 and cfg == ref["config"]
    from triton_tagi.checkpoint import net_state

    _same_state(net_state(net), ref["net_state"])


def test_checkpoint_written_here_matches_the_reference_layout(tmp_path):
    ref = torch.load(GOLDEN / "ref_checkpoint.pt", weights_only=False)
    net = _build()
    from triton_tagi.checkpoint import restore_net_state

    restore_net_state(net, ref["net_state"])
    run = TT.RunDir("synthetic", "small", "tagi", base=str(tmp_path))
    path = run.save_checkpoint(net, 7, ref["config"])
    assert path == run.checkpoints / "epoch_0007.pt"
    mine = torch.load(path, weights_only=False)
    assert mine.keys() == ref.keys() and mine["epoch"] == 7 and mine["config"] == ref["config"]
    _same_state(mine["net_state"], ref["net_state"])
    # and back: a fresh network restored from it by RunDir.load_checkpoint
    other = _build()
    assert run.load_checkpoint(other) == 7
    from triton_tagi.checkpoint import net_state

    _same_state(net_state(other), ref["net_state"])


def test_run_directory_layout_and_metrics(tmp_path):
    run = TT.RunDir("cifar10", "resnet18", "tagi", base=str(tmp_path))
    assert run.path.parent == tmp_path and run.path.name.startswith("cifar10_resnet18_tagi_")
    assert run.checkpoints.is_dir() and run.figures.is_dir()
    run.save_config({"batch": 128, "sigma_v": 0.05})
    assert json.loads(run.config_json.read_text()) == {"batch": 128, "sigma_v": 0.05}
    run.append_metrics(1, loss=0.123456789, acc=0.5)
    run.append_metrics(2, loss=0.1, acc=0.75)
    rows = list(csv.DictReader(open(run.metrics_csv)))
    assert rows == [{"epoch": "1", "loss": "0.123457", "acc": "0.5"},
                    {"epoch": "2", "loss": "0.1", "acc": "0.75"}]
    try:
        run.load_checkpoint(_build())
        raise AssertionError("expected FileNotFoundError")
    except FileNotFoundError:
        pass
