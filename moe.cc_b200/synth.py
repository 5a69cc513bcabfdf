"""Seeded synthetic Qwen3-30B-A3B-shaped MoE layers (harness helpers).

Every tensor is drawn from the counter-based normal stream of
moe_synth_normal_{host,dev} (splitmix64 -> Box-Muller), so host and device
builds of the same layer agree. Seeds: tensor `tid` of layer `layer` under
base seed `seed` uses stream seed*1_000_003 + layer*1009 + tid, with
tid = 0 router, 1 router bias, 2+3e gate e, 3+3e up e, 4+3e down e.
Expert weights ~ N(0, 0.02) quantised rowwise (export.py:23-36 semantics),
router ~ N(0, 0.02), bias ~ N(0, 1) when requested.
"""
import moe_cuda as mc

QWEN3 = dict(E=128, D=2048, F=768, topk=8)


def stream_seed(seed, layer, tid):
    return (seed * 1_000_003 + layer * 1009 + tid) & ((1 << 64) - 1)


def make_layer_dev(torch, seed, layer, E, D, F, dtype, bias=False, device="cuda"):
    """Build one layer on the GPU: fp32 normals -> device quantiser. Returns a
    dict of torch CUDA tensors in the moe_cuda.upload_layer layout."""
    f32 = torch.float32
    L = {"dtype": dtype}
    rw = torch.empty(E, D, dtype=f32, device=device)
    mc.synth_normal_dev(stream_seed(seed, layer, 0), rw, 0.02)
    L["router_w"] = rw
    if bias:
        b = torch.empty(E, dtype=f32, device=device)
        mc.synth_normal_dev(stream_seed(seed, layer, 1), b, 1.0)
        L["router_b"] = b
    qdt = torch.int8 if dtype == mc.Q8 else torch.uint8
    shapes = {"g": (F, D), "u": (F, D), "d": (D, F)}
    for j, nm in enumerate("gud"):
        rows, cols = shapes[nm]
        qcols = cols if dtype == mc.Q8 else cols // 2
        q = torch.empty(E, rows, qcols, dtype=qdt, device=device)
        s = torch.empty(E, rows, dtype=f32, device=device)
        tmp = torch.empty(rows, cols, dtype=f32, device=device)
        for e in range(E):
            mc.synth_normal_dev(stream_seed(seed, layer, 2 + 3 * e + j), tmp, 0.02)
            mc.quantize_rowwise_dev(tmp, q[e], s[e], dtype)
        L[nm + "q"], L[nm + "s"] = q, s
    return L


def make_tokens_dev(torch, seed, T, D, device="cuda"):
    x = torch.empty(T, D, dtype=torch.float32, device=device)
    mc.synth_normal_dev(stream_seed(seed, 0, 0x7FFFFFFF), x, 1.0)
    return x
