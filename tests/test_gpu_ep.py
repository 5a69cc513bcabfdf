"""GPU: expert parallelism over 2 ranks (moe_ffn_partial + exchange +
moe_ffn_combine) reproduces the single-device oracle result bit for bit:
every slot is computed by exactly one rank, so the sum over ranks is exact."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("dt,T", [(2, 16), (2, 40)])
def test_expert_parallel_two_ranks_matches_oracle(tmp_path, dt, T):
    out = str(tmp_path / "ep.npz")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(29500 + T),
           os.path.join(HERE, "ep_worker.py"), out, str(T), str(dt)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    from oracle.oracle import Port
    z = np.load(out)
    L = {"dtype": dt, "topk": 8, "router_b": None}
    for k in ("router_w", "gq", "gs", "uq", "us", "dq", "ds"):
        L[k] = z[k]
    ref, _, _, _ = Port().moe_block(z["xn"], z["xa"], L)
    assert np.array_equal(z["out"], ref)
