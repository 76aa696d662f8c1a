"""Shared pytest setup.

* registers the `gpu` marker (tests that need a B200; run with -m gpu);
* puts the repo root (oracle/) and triton-metal_b200/ (b200kern) on sys.path;
* builds libb2.so in-tree if it is missing (nvcc cross-compiles without a GPU).
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "triton-metal_b200")
for p in (REPO, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def _ensure_built():
    lib = os.path.join(PKG_ROOT, "b200kern", "libb2.so")
    if not os.path.exists(lib):
        sys.path.insert(0, os.path.join(PKG_ROOT, "csrc"))
        import build as _b  # csrc/build.py
        _b.build()
    return lib


_ensure_built()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    assert (major, minor) == (10, 0), f"libb2.so is built for sm_100a, device is sm_{major}{minor}"
    return torch.device("cuda:0")


def golden(name):
    import numpy as np
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))
