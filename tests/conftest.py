import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda_ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    import qppocr_b200 as q

    return q.CudaContext.open(0)
