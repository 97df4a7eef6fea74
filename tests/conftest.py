import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import pyoracle
    pyoracle.build()
    return pyoracle


@pytest.fixture(scope="session")
def navlib():
    from neuraval_b200 import build, native
    build.build()
    return native.load()


@pytest.fixture(scope="session")
def gpu_sampler(navlib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    from neuraval_b200.sampler import CudaTokenSampler
    s = CudaTokenSampler(device=0, max_rows=1024, max_vocab=262144, max_history=4096)
    yield s
    s.close()
