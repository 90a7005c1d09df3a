import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(os.path.join(GOLDEN, "lib_c_vectors.npz")))


@pytest.fixture(scope="session")
def block_golden():
    return dict(np.load(os.path.join(GOLDEN, "rac_torch_block.npz")))


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.orc()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    from rac_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")
