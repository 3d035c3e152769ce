"""Test configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs everywhere (oracle vs golden vectors, host logic, C-ABI
loading).  ``-m gpu`` needs an SM100 (B200) device and calls the native
library; those tests are skipped, not silently passed, when no GPU is present.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"

# FlashInfer (the reference's NVFP4 backend, used only as the GPU checker)
# loads its prebuilt modules from the in-tree cache that
# tests/golden/build_flashinfer_reference.py builds.
os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", str(ROOT / "tests" / ".flashinfer_ref"))
os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an SM100 (B200) CUDA device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        have_gpu = torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:  # pragma: no cover
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="no SM100 CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN / "fp8_golden.npz"))
