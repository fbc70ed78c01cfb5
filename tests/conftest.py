"""Shared test setup.

* registers the ``gpu`` marker (tests that need a CUDA device) and ``slow``;
* puts the repo root (for ``oracle``) and ``pyramid-forcing_b200`` (for the
  ``pyramidkv`` package) on sys.path;
* seeds numpy/torch per test.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "pyramid-forcing_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(autouse=True)
def _seed():
    np.random.seed(0)
    try:
        import torch
        torch.manual_seed(0)
    except ImportError:  # pragma: no cover
        pass


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test run without a visible CUDA device")
    from pyramidkv import _ops
    assert _ops.available(), "the adahead library must load on a CUDA machine"
    return torch.device("cuda:0")


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name))
