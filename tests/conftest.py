"""Shared pytest setup: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs on any machine (oracle vs golden vectors, host logic, the
C-ABI library's exports); ``-m gpu`` needs a CUDA device and calls the CUDA
kernels through the C-ABI.
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "vllm-expert-pager_b200")
for p in (PKG_ROOT, REPO, os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs the sm_100a kernels)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
