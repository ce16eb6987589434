"""Shared fixtures.  Tests marked ``gpu`` need a CUDA device (B200); the rest
run on CPU and cover the oracle against the golden fixtures, host logic, the
C ABI's host-side surface and gloo multi-process shard logic."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run with -m gpu)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str) -> dict:
    path = os.path.join(GOLDEN, name + ".npz")
    with np.load(path, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture
def device():
    import torch
    return torch.device("cuda")


@pytest.fixture(scope="session")
def ba():
    """The batchaug_b200 package (CUDA library loaded)."""
    import batchaug_b200
    return batchaug_b200
