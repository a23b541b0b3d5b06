"""Shared test configuration.

Markers: ``gpu`` -- needs a CUDA device (B200) and the built library; these are
the parity tests proper and call the library through its C ABI.  Everything
unmarked runs on a CPU-only machine.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "nova-wino-amd_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libnova_winograd.so")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def seed():
    # Same autouse seeding as the reference suite (tests/test_correctness.py:29-31).
    import torch
    torch.manual_seed(42)
