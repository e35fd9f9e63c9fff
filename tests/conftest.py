"""Shared pytest configuration.

Tests that need a B200 are marked ``gpu``; without a GPU they are skipped. CPU tests
use one torch thread (CPU results may depend on the thread count, as the reference's
suite notes).
"""

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).parent))

torch.set_num_threads(1)

HAS_CUDA = torch.cuda.is_available()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (a B200)")


def pytest_collection_modifyitems(config, items):
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords and not HAS_CUDA:
            item.add_marker(skip)
