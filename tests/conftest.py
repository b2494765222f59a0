"""Shared pytest configuration.

Markers:
  gpu   needs a CUDA device (a B200) and the built native library; deselect
        with ``-m "not gpu"`` on CPU-only machines.
  slow  multi-process or long-running CPU tests.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the native library")
    config.addinivalue_line("markers", "slow: multi-process or long-running test")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
