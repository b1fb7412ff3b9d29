import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU (runs through libmxq.so)")


@pytest.fixture(scope="session")
def ctx():
    import torch
    from cpu_model_b200 import mx
    assert torch.cuda.is_available(), "GPU test collected without a GPU"
    c = mx.MXContext(0)
    yield c
    c.close()
