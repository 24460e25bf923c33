"""Test configuration.

Tiers: ``-m "not gpu"`` runs here without a GPU (the oracle against the reference's golden
vectors, host-side logic, the C ABI's exports and refusals); ``-m gpu`` runs on a B200 and
compares the CUDA kernels, called through the C ABI, with the oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device that runs sm_100a (B200)")


@pytest.fixture(scope="session")
def cuda():
    """The torch module with a usable B200; a GPU test without one fails rather than skips."""
    import torch

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"sm_100a kernels need a cc 10.0 device, got {major}.{minor}"
    return torch


@pytest.fixture(scope="session")
def ops(cuda):
    from shipinfer_b200 import NativeImageOps

    return NativeImageOps(device_index=0)


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle

    oracle.build()
    return oracle
