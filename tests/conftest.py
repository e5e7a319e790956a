"""Test configuration: the `gpu` marker selects tests that need a B200 (sm_100a).

`python -m pytest tests -m "not gpu"` runs the CPU suite (oracle vs golden
vectors, host logic, C-ABI exports, gloo multi-process tests);
`python -m pytest tests -m gpu` runs the CUDA parity tests, which call the
sm_100a library through its C ABI and compare against the CPU oracle.
"""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100a device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
