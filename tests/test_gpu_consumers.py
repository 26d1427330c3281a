"""Every quantized decode consumer stays parity-checked whatever the default
dispatch picks: the tensor-core tile kernel (tc, batch-1 D=128 q4+/q8+), the
grouped-query tensor-core consumer (mma) and the integer dot-product
consumer (dp) each run batch-1 and grouped-query cases against the oracle,
in a fresh process with VOLTATTN_CONSUMER set (tests/consumer_check.py)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("consumer", ["tc", "mma", "dp"])
def test_consumer(consumer):
    env = dict(os.environ, VOLTATTN_CONSUMER=consumer)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "consumer_check.py")], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
