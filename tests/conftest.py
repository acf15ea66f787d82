import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


@pytest.fixture(scope="session")
def ctx():
    """One library context on cuda:0 for the GPU tests (fails loudly without the library)."""
    import torch
    torch.cuda.set_device(0)
    torch.cuda.init()
    import vxg_b200
    c = vxg_b200.Context()
    yield c
    c.close()
