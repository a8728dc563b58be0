import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    # a run that selects gpu tests on a machine without a GPU should fail loudly,
    # not skip: the product has no CPU fallback
    pass


@pytest.fixture(scope="session")
def gpu_ctx():
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    from pesti_b200 import kq
    ctx = kq.Context(0)
    yield ctx
    ctx.close()
