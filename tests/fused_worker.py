"""Child process for tests/test_gpu_fused.py: runs moe_ffn on the
Qwen3-30B-A3B layer shape (Q8, seeded synthetic weights) for several token
counts and saves outputs and top-k. The decode kernel selection
(MOE_FUSED: 0 = gate/up and down as two kernels, 2 = the fused persistent
kernel for every decode size) is read once per process, hence a child."""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "moe.cc_b200"))
import moe_cuda as mc  # noqa: E402
import synth as sy  # noqa: E402


def main():
    out, ts = sys.argv[1], [int(v) for v in sys.argv[2].split(",")]
    dt = int(sys.argv[3]) if len(sys.argv) > 3 else 2
    mc.init(0)
    Ld = sy.make_layer_dev(torch, 1, 0, 128, 2048, 768, dt)
    mc.upload_layer(0, Ld, device_arrays=True)
    res = {}
    for T in ts:
        xn = sy.make_tokens_dev(torch, 700 + T, T, 2048)
        xo = sy.make_tokens_dev(torch, 800 + T, T, 2048)
        idx = torch.empty(T, 8, dtype=torch.int32, device="cuda")
        p = torch.empty(T, 8, device="cuda")
        for rep in range(3):            # repeated calls: the work counters must reset
            x = xo.clone()
            mc.moe_ffn_dev(0, xn, x, idx, p)
            torch.cuda.synchronize()
            mc.check_status()
            if rep == 0:
                first = x.cpu().numpy()
            else:
                assert np.array_equal(first, x.cpu().numpy()), f"T={T}: call {rep} differs"
        res[f"out_{T}"] = first
        res[f"idx_{T}"] = idx.cpu().numpy()
        res[f"xn_{T}"] = xn.cpu().numpy()
        res[f"xo_{T}"] = xo.cpu().numpy()
    np.savez(out, **res)


if __name__ == "__main__":
    main()
