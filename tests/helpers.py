"""Shared builders for the tests: seeded layers in the upload layout."""
import os

import numpy as np

import moe_cuda as mc
from oracle.oracle import quantize_q4, quantize_q8

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def synth(seed, n, std):
    return mc.synth_normal_host(seed, n, std)


def quant(dt):
    return quantize_q8 if dt == 2 else quantize_q4


def small_layer(E, D, F, dt, bias, seed_base=0):
    """Same construction as tests/golden/make_golden.small_layer (numpy quantiser,
    pinned bit-exact to export.py by the golden vectors)."""
    L = {"dtype": dt, "topk": 8,
         "router_w": synth(30 + dt + seed_base, E * D, 0.02).reshape(E, D)}
    L["router_b"] = synth(31 + dt + seed_base, E, 1.0) if bias else None
    shapes = {"g": (F, D), "u": (F, D), "d": (D, F)}
    for j, nm in enumerate("gud"):
        rows, cols = shapes[nm]
        ss, qs = [], []
        for e in range(E):
            w = synth(1000 * dt + 3 * e + j + 7919 * seed_base, rows * cols, 0.02).reshape(rows, cols)
            s, q = quant(dt)(w)
            ss.append(s); qs.append(q)
        L[nm + "s"] = np.ascontiguousarray(np.stack(ss))
        L[nm + "q"] = np.ascontiguousarray(np.stack(qs))
    return L


def layer_to_torch(L, torch):
    out = {}
    for k, v in L.items():
        out[k] = torch.from_numpy(v).cuda() if isinstance(v, np.ndarray) else v
    return out


def layer_to_numpy(Ld):
    out = {}
    for k, v in Ld.items():
        out[k] = v.cpu().numpy() if hasattr(v, "cpu") else v
    return out
