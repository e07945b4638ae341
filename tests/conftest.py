"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200 for the performance-sized
cases); everything else runs on the CPU. The CPU suite covers the oracle
against the reference's golden vectors, the host-side logic, and that the
C-ABI library loads and exports every symbol ``include/fracture_b200.h``
declares.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on the CPU")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    here = os.path.join(ROOT, "tests", "golden")
    return [np.load(os.path.join(here, f"fixture_prompt{p}.npz")) for p in (0, 1)]
