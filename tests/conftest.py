import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.build_oracle_lib()
    return o


@pytest.fixture(scope="session")
def cuda_dev():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device (run with -m 'not gpu' on CPU)"
    from nki_moe_7013_b200 import _C

    _C.lib()
    return torch.device("cuda:0")
