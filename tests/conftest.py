"""Shared pytest configuration: the `gpu` marker and the repository root on sys.path."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a); run with -m gpu")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for GPU tests; the library must be loadable (no silent fallback)."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device visible")
    import rocmkernels_b200

    rocmkernels_b200.lib()  # raises if the sm_100a library was not built
    return torch.device("cuda:0")
