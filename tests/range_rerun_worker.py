"""Child process for tests/test_gpu_range_rerun.py: host-pointer moe_ffn on
inputs beyond the fast kernels' integer range (Q8 |x| >= 258, Q4
trunc(7x) outside [-128, 127]), checked against the oracle. MOE_RANGE_RERUN
is read once per process, hence a child per setting; argv[1] is 1 when it
is set."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "moe.cc_b200"), HERE):
    sys.path.insert(0, p)
import moe_cuda as mc  # noqa: E402
from helpers import small_layer, synth  # noqa: E402
from oracle.oracle import Port  # noqa: E402


def main():
    rerun = sys.argv[1] == "1"
    mc.init(0)
    port = Port()
    for dt, scale in ((2, 400.0), (3, 40.0)):
        L = small_layer(16, 256, 256, dt, bias=(dt == 3), seed_base=9)
        mc.upload_layer(700 + dt, L)
        for T in (3, 8):
            xn = synth(60 + T, T * 256, 1.0).reshape(T, 256) * np.float32(scale)
            xa = synth(61 + T, T * 256, 1.0).reshape(T, 256)
            for call in range(2):
                try:
                    xo, idx, p = mc.moe_ffn_host(700 + dt, xn, xa)
                except mc.MoeError as e:
                    assert not rerun and e.code == mc.MOE_ERR_RANGE, str(e)
                    continue
                assert rerun, "out-of-range input computed without the re-run"
                ref, ref_idx, ref_p, _ = port.moe_block(xn, xa, L)
                assert np.array_equal(idx, ref_idx) and np.array_equal(p, ref_p)
                tol = 1e-4 * float(np.abs(ref).max())
                assert float(np.abs(xo - ref).max()) <= tol, f"dtype {dt} T={T} call {call}"
        mc.free_layer(700 + dt)
    print("ok")


if __name__ == "__main__":
    main()
