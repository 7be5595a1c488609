"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on CPU."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on a B200 with -m gpu)")


@pytest.fixture(scope="session", autouse=True)
def native_libraries() -> None:
    """Build (if stale) the product library and the oracle's C checker once per session."""
    from oracle import stream
    from warpshift_b200 import build

    build.build()
    stream.build()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)
