"""Host-pointer moe_ffn on activations beyond the fast kernels' integer range:
without MOE_RANGE_RERUN the call reports MOE_ERR_RANGE; with it, the experts
are recomputed with exact int32 activations and match the oracle.

Off by default: set MOE_TEST_RANGE_RERUN=1 to run it (the switch itself stays
off by default until this test has passed on a GPU)."""
import os
import subprocess
import sys

import pytest

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("MOE_TEST_RANGE_RERUN") != "1",
                                 reason="set MOE_TEST_RANGE_RERUN=1 to run the exact re-run comparison")]
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("rerun", ["0", "1"])
def test_range_rerun(rerun):
    env = dict(os.environ, MOE_RANGE_RERUN=rerun)
    r = subprocess.run([sys.executable, os.path.join(HERE, "range_rerun_worker.py"), rerun], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-3000:]
