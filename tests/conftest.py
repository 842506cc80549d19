import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Build the oracle (CPU checker) and the CUDA library once per session."""
    from oracle import oracle
    oracle.build()
    from common_b200 import build
    build.build()
    yield


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
