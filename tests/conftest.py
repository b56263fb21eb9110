"""Shared pytest setup: the `gpu` marker, the in-tree native build, daemon fixtures."""
from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "gpu_extended: long GPU property tests; run with -m gpu_extended "
                            "(skipped without a GPU, not part of -m gpu)")


@pytest.fixture(scope="session", autouse=True)
def native_build():
    """Make sure libugdr.so and the binaries exist (builds them once if missing or stale)."""
    from ugdr_b200.utils.build import build

    build()
    yield


@pytest.fixture
def cpu_daemon():
    from ugdr_b200 import verbs as V

    d = V.Daemon(gpus=0)
    yield d
    d.stop()


def gpu_count() -> int:
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0
