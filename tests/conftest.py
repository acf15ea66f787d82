import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


@pytest.fixture
def ctx():
    """A fresh library context on cuda:0 per test (fails loudly without the library), so a
    context poisoned by one test's failure does not take the others down."""
    import torch
    torch.cuda.set_device(0)
    torch.cuda.init()
    import vxg_b200
    c = vxg_b200.Context()
    yield c
    c.close()
