"""Test configuration: the ``gpu`` marker and shared helpers.

Tests marked ``gpu`` need a CUDA device (a B200) and the built C library;
everything else runs on CPU.  ``pytest -m "not gpu"`` is the CPU suite.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and libldb200.so")


@pytest.fixture(scope="session")
def cuda_device():
    """The CUDA device for GPU tests; fails (never skips) when a gpu test has no GPU."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a test marked gpu ran without a CUDA device")
    return torch.device("cuda:0")
