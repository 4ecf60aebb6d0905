import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def built_lib():
    """Path of libks_b200.so, building it when it is missing or stale and nvcc exists."""
    from kernelswift_b200 import build

    if not build.up_to_date():
        try:
            build.build()
        except RuntimeError:
            if not os.path.exists(build.OUT):
                raise
    return build.OUT


@pytest.fixture(scope="session")
def cuda_ok(built_lib):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def load_golden(name):
    import numpy as np

    return np.load(os.path.join(GOLDEN, name + ".npz"))
