import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture
def cpu_threads():
    import torch
    old = torch.get_num_threads()
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    yield
    torch.set_num_threads(old)
