"""Child process of tests/test_gpu_wait_expiry.py (one GPU).

Makes the expert-parallel flag waits run out without faulting anything: a
group of two ranks in which both entries of the connection table are this
process's own buffer (loopback), so the flags of "rank 1" are never raised.
moe_ffn_ep must return after the time limit (MOE_EP_WAIT_MS, set short by the
parent), moe_cuda_check_status must report the timeout, a fresh
ep_setup/ep_connect must work again (and time out again, cleanly), and after a
shutdown the library must compute a normal call correctly on the same GPU.
"""
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "moe.cc_b200"), HERE):
    sys.path.insert(0, p)
import moe_cuda as mc  # noqa: E402
from helpers import small_layer, synth  # noqa: E402
from oracle.oracle import Port  # noqa: E402


def one_timed_out_call(L, T):
    h = mc.ep_setup(T, 256, 8)
    mc.ep_connect([h, h])                  # loopback: "rank 1" is this buffer too
    xn = torch.from_numpy(synth(61, T * 256, 1.0).reshape(T, 256)).cuda()
    xo = torch.zeros(T, 256, device="cuda")
    t0 = time.perf_counter()
    mc.moe_ffn_ep(7, xn, xo)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    try:
        mc.check_status()
        raise AssertionError("the flag waits did not report a timeout")
    except mc.MoeError as e:
        assert e.code == mc.MOE_ERR_CUDA and "wait" in str(e), str(e)
    return dt


def main():
    mc.init(0, 2, 0)
    L = small_layer(16, 256, 256, 2, bias=False, seed_base=9)
    mc.upload_layer(7, L)
    limit = float(os.environ["MOE_EP_WAIT_MS"]) / 1e3
    for _ in range(2):                     # fresh setup / connect after an expiry
        dt = one_timed_out_call(L, 4)
        # two waits (dispatch, combine), each bounded by the limit
        assert dt < 2 * limit + 2.0, f"the call took {dt:.2f} s"
    mc.shutdown()
    # the context is intact: a normal call on the same GPU is exact
    mc.init(0)
    mc.upload_layer(8, L)
    xn = synth(62, 8 * 256, 1.0).reshape(8, 256)
    xa = synth(63, 8 * 256, 1.0).reshape(8, 256)
    xo, idx, _ = mc.moe_ffn_host(8, xn, xa)
    ref, ref_idx, _, _ = Port().moe_block(xn, xa, L)
    assert np.array_equal(idx, ref_idx) and np.array_equal(xo, ref)
    print("wait expiry ok")


if __name__ == "__main__":
    main()
