"""Child process for tests/test_gpu_e2e_graph.py: host-pointer moe_ffn calls
(stream NULL) on two Qwen3-shaped layers, Q8 and Q4, for several token
counts, rotating over input buffers and layers as bench.py's e2e leg does,
and saves every call's outputs. MOE_E2E_GRAPH is read once per process,
hence a child per setting."""
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
    out = sys.argv[1]
    mc.init(0)
    for lid, dt in ((0, 2), (1, 3)):
        Ld = sy.make_layer_dev(torch, 1, lid, 128, 2048, 768, dt)
        mc.upload_layer(lid, Ld, device_arrays=True)
        del Ld
    torch.cuda.synchronize()
    res = {}
    for T in (1, 4, 16, 64):
        xs = [mc.synth_normal_host(900 + 10 * T + i, T * 2048, 1.0).reshape(T, 2048) for i in range(3)]
        xa = [mc.synth_normal_host(950 + 10 * T + i, T * 2048, 1.0).reshape(T, 2048) for i in range(3)]
        for call in range(6):                # two eager-then-graph keys, three buffer sets
            lid = call % 2
            xo, idx, p = mc.moe_ffn_host(lid, xs[call % 3], xa[call % 3])
            res[f"x_{T}_{call}"], res[f"i_{T}_{call}"], res[f"p_{T}_{call}"] = xo, idx, p
    np.savez(out, **res)


if __name__ == "__main__":
    main()
