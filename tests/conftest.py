import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libcmol.so")
    config.addinivalue_line("markers", "slow: long-running")


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    if not has_gpu():
        pytest.skip("no CUDA device")
    import torch
    torch.cuda.init()
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def tmpdir_models(tmp_path_factory):
    return tmp_path_factory.mktemp("models")
