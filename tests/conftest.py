import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def ctx():
    """One lalb context on cuda:0 for the whole GPU session."""
    import torch

    import lalmodel_b200 as lb

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    c = lb.Context(0)
    yield c
    torch.cuda.synchronize()
    assert c.device_status() == 0, "a bounded device wait expired during the session"
    c.close()
