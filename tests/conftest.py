"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any machine (oracle vs golden fixtures, host logic, C-ABI
loading, distributed host logic on gloo).  `-m gpu` needs a CUDA GPU and runs the
parity tests through the C ABI.
"""

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / "tests"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU; runs the sm_100a kernels")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
