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


def assert_matches_port(out, ref, T, xn):
    """The layer tolerance 1e-4*max|y| (north_star's bar), then bit-exact
    equality (integer dots, the reference's float order, libc's expf)."""
    err = float(np.abs(out - ref).max())
    assert err <= 1e-4 * float(np.abs(ref).max()), f"max-abs {err}"
    assert np.array_equal(out, ref), f"only {float(np.mean(out == ref)):.6f} bit-identical (T={T})"


@pytest.mark.parametrize("dt,T,inputs", [(2, 16, "normal"), (2, 40, "normal"), (2, 256, "normal"),
                                         (2, 16, "big"), (3, 40, "big")])
def test_expert_parallel_two_ranks_matches_oracle(tmp_path, dt, T, inputs):
    out = str(tmp_path / "ep.npz")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(29500 + T + 7 * dt + (50 if inputs == "big" else 0)),
           os.path.join(HERE, "ep_worker.py"), out, str(T), str(dt), "nccl", inputs]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    from oracle.oracle import Port
    z = np.load(out)
    L = {"dtype": dt, "topk": 8, "router_b": None}
    for k in ("router_w", "gq", "gs", "uq", "us", "dq", "ds"):
        L[k] = z[k]
    ref, _, _, _ = Port().moe_block(z["xn"], z["xa"], L)
    assert_matches_port(z["out"], ref, T, z["xn"])


@pytest.mark.parametrize("dt,T,mode,inputs", [(2, 16, "fused", "normal"), (3, 40, "fused", "normal"),
                                              (2, 256, "fused", "normal"), (2, 16, "fused", "big"),
                                              (3, 40, "fused", "big"), (2, 16, "skip", "normal")])
def test_fused_expert_parallel_two_gpus_matches_oracle(tmp_path, dt, T, mode, inputs):
    """moe_ffn_ep: the down GEMM stores slot rows into the owning rank's
    receive buffer over NVLink and the combine waits on the ranks' flags.
    "big": out-of-range tokens, recomputed by the experts' owners' exact
    fix-up pass. "skip": rank 1 first leaves a call out; rank 0's bounded
    waits run out and report it, then a fresh setup works. Needs one GPU per
    rank (ranks spin on one another)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("the fused exchange needs one GPU per rank (2 GPUs)")
    out = str(tmp_path / "epf.npz")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1",
           "--master-port", str(29700 + T + dt + (40 if inputs == "big" else 0) + (80 if mode == "skip" else 0)),
           os.path.join(HERE, "ep_worker.py"), out, str(T), str(dt), mode, inputs]
    # the skip case: short flag waits, and no NVLink multicast in NCCL while a
    # rank sits a call out
    env = dict(os.environ, MOE_EP_WAIT_MS="100", NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    from oracle.oracle import Port
    z = np.load(out)
    L = {"dtype": dt, "topk": 8, "router_b": None}
    for k in ("router_w", "gq", "gs", "uq", "us", "dq", "ds"):
        L[k] = z[k]
    ref, _, _, _ = Port().moe_block(z["xn"], z["xa"], L)
    assert_matches_port(z["out"], ref, T, z["xn"])
