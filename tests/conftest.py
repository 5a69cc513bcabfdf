import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "moe.cc_b200"), os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 and the built libmoe_cuda.so")


@pytest.fixture(scope="session")
def gpu():
    """Initialise libmoe_cuda on cuda:0 once per session."""
    import moe_cuda as mc
    mc.init(0)
    yield mc
