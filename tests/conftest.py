import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("ltc-cuda_b200", ""):
    path = os.path.join(REPO, sub) if sub else REPO
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(autouse=True)
def no_expired_device_waits(request):
    """Every GPU test must leave the library's bounded in-kernel waits unexpired
    (cluster exchange, TMA chunk arrivals): an expiry means a launch gave up waiting."""
    if request.node.get_closest_marker("gpu") is None:
        yield
        return
    import ltc_cuda
    before = ltc_cuda.wait_timeouts()
    yield
    assert ltc_cuda.wait_timeouts() == before, "a bounded in-kernel wait expired"
