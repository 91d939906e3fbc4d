import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import __graft_entry__ as G  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (run with -m gpu)")


@pytest.fixture(scope="session")
def O():
    """The CPU oracle (test infrastructure)."""
    return G.oracle()


@pytest.fixture(scope="session")
def P():
    """The product package (libdcinfer.so behind ctypes)."""
    return G.package()


@pytest.fixture(scope="session")
def comp(P):
    """A gated compute core on cuda:0, launching on torch's current stream."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a -m gpu test ran without a CUDA device")
    torch.cuda.init()
    c = P.init_compute(0, stream=torch.cuda.current_stream())
    yield c
    c.close()
