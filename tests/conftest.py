"""pytest configuration: the `gpu` marker and repository imports.

Tests marked ``gpu`` need a B200 and the built ``libaios_b200.so``; the rest run
on any CPU machine (``pytest -m "not gpu"``).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and the native library")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("GPU tests need a CUDA device")
    return torch.device("cuda", 0)
