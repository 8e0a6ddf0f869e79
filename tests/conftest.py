import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("", "oracle", "cuda-repo_b200", "tests"):
    p = os.path.join(REPO, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100 (got sm_{major}{minor})")
    return torch.device("cuda:0")


@pytest.fixture
def tuning():
    """spmm24.set_tuning for one test, reset to the automatic picker after it."""
    import spmm24

    yield spmm24.set_tuning
    spmm24.reset_tuning()
