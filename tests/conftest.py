import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def golden():
    import json
    import numpy as np
    g = os.path.join(ROOT, "tests", "golden")
    with open(os.path.join(g, "golden.json")) as fh:
        digests = json.load(fh)
    return {
        "digests": digests,
        "selftest": np.load(os.path.join(g, "selftest_ref.npz")),
        "edge": np.load(os.path.join(g, "edge_quant.npz")),
    }


@pytest.fixture(autouse=True)
def _no_silent_device_errors(request):
    """Every GPU test ends with the library's device error word clear: a
    bounded wait that gave up inside a kernel fails the test that launched it
    (tests that provoke one on purpose read and clear the word themselves)."""
    yield
    if request.node.get_closest_marker("gpu") is None or "voltattn_b200" not in sys.modules:
        return
    import torch
    if not torch.cuda.is_available():
        return
    va = sys.modules["voltattn_b200"]
    torch.cuda.synchronize()
    err = va.device_error()
    assert err == 0, f"a kernel of this test reported device error {err} (a bounded wait gave up)"
