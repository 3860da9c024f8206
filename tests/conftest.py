"""Shared pytest configuration.

Markers: ``gpu`` (needs a CUDA device and the built sm_100a library) and
``slow``. The repository root and the host package directory are put on
``sys.path`` so that ``import oracle`` and ``import triton_tagi`` resolve to the
copies in this repository.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "triton-tagi_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU and the built sm_100a library")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_runtest_setup(item):
    if item.get_closest_marker("gpu"):
        import torch

        if not torch.cuda.is_available():
            pytest.skip("CUDA not available")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    cache = {}

    def get(name):
        if name not in cache:
            cache[name] = np.load(GOLDEN / f"{name}.npz")
        return cache[name]

    return get
