"""Shared pytest setup: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a CUDA device and the built extension; everything
else runs on the CPU (the oracle against the reference's golden vectors, the
host-side validation, the C-ABI export table, gloo multi-rank logic).
"""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "01-glm53-ascend_b200"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built extension")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
