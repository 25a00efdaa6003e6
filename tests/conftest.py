"""Shared pytest configuration.

Marker ``gpu``: the test needs a CUDA device (a B200 for the sm_100a kernels).
The CPU tier runs with ``-m "not gpu"``; the GPU tier with ``-m gpu``.
"""

from __future__ import annotations

import pytest
import torch


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a kernels)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
