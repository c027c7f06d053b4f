"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any host (oracle, C-ABI loading and host-side
validation, planner, Python argument checks, gloo multi-process logic);
`-m gpu` needs an sm_100 device and the in-tree binaries.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "tma-depthwise-conv_b200")
for p in (PKG, os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 CUDA device")


def _cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
