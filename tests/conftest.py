import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built_artifacts():
    """Compile libkat_rational.so and the C oracle if their sources are newer."""
    from rational_kat_cu_b200 import _build
    from oracle import build as oracle_build

    if _build.is_stale():
        _build.build()
    oracle_build.build()
    yield


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    return torch.device("cuda", 0)
