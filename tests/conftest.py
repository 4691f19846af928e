import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


@pytest.fixture(autouse=True)
def _reset_backend():
    from afd_demo_b200.parallel.dist import DistributedContext
    from afd_demo_b200.utils import device as devmod

    yield
    DistributedContext.reset()
    devmod.reset_backend()
