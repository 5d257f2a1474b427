import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.lib()
    return O


@pytest.fixture(scope="session")
def cuda():
    import torch

    assert torch.cuda.is_available(), "GPU test selected but no CUDA device is visible"
    import rapier_b200

    rapier_b200.load()  # fails loudly when the library is missing

    # the C-ABI requires an explicit stream (as the reference's native_mmvq does): run every test on one
    torch.cuda.set_stream(torch.cuda.Stream(device=0))
    return torch.device("cuda:0")
