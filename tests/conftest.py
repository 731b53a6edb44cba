import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def port():
    import oracle

    return oracle.port()


@pytest.fixture(scope="session")
def ref():
    import oracle

    if not oracle.ref_available():
        pytest.skip("reference CPU build (oracle/_ref) not present on this machine")
    return oracle.ref()


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mini_llama_b200 as mlb

    assert mlb.CudaQuantBuilt()
    return torch


def golden_path(name):
    return os.path.join(ROOT, "tests", "golden", name)
