import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")
    config.addinivalue_line("markers", "slow: full-size workload")


@pytest.fixture(scope="session")
def restated():
    from oracle.oracle import Restated
    return Restated()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import REFERENCE_SO, Reference
    if not os.path.exists(REFERENCE_SO):
        pytest.skip("oracle/_ref/libtvref.so not built (reference sources absent)")
    return Reference()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    path = os.path.join(ROOT, "tests", "golden", "golden.npz")
    return dict(np.load(path, allow_pickle=False))


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from ternative_b200 import load
    load()   # fails loudly when libtvb200.so is missing
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def backend(cuda):
    from ternative_b200 import CUDABackend
    return CUDABackend()
