"""GPU: the expert-parallel flag waits are bounded by time and leave the
library usable. The flags that are waited on are never raised (a loopback
group in one process, no second rank and no fault); see wait_expiry_worker.py."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_flag_waits_expire_and_recover():
    env = dict(os.environ, MOE_EP_WAIT_MS="50")
    r = subprocess.run([sys.executable, os.path.join(HERE, "wait_expiry_worker.py")], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    assert "wait expiry ok" in r.stdout
