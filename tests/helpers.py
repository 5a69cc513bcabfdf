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


# ---- the reference's .bin weight file (export.py _save_tensor, :8-21) ----
BIN_MAGIC = b"QW3W\x00\x01"
_BIN_DTYPE = {np.dtype(np.float32): 0, np.dtype(np.float16): 1,
              np.dtype(np.int8): 2, np.dtype(np.uint8): 3}


def write_bin(path, tensors, count=None):
    """Writes (name, ndarray) records in the .bin layout; pinned byte for byte
    to the reference's writer by tests/golden/layer_ref.bin."""
    import struct
    with open(path, "wb") as f:
        f.write(BIN_MAGIC)
        f.write(struct.pack("<I", len(tensors) if count is None else count))
        for name, a in tensors:
            a = np.ascontiguousarray(a)
            nb = name.encode()
            f.write(struct.pack("<I", len(nb)) + nb)
            f.write(struct.pack("<II", _BIN_DTYPE[a.dtype], a.ndim))
            f.write(struct.pack("<" + "I" * a.ndim, *a.shape))
            f.write(a.tobytes())


def layer_records(L, layer, router_name="mlp.gate.weight"):
    """One quantised MoE layer as .bin records, in the exporter's order
    (router, bias, then per projection .scale before .q8/.q4, export.py:197-206)."""
    q = "q8" if L["dtype"] == 2 else "q4"
    pre = f"model.layers.{layer}."
    recs = [(pre + router_name, np.asarray(L["router_w"], np.float32))]
    if L.get("router_b") is not None:
        recs.append((pre + "mlp.gate.bias", np.asarray(L["router_b"], np.float32)))
    E = L["router_w"].shape[0]
    for e in range(E):
        for nm, proj in (("g", "gate_proj"), ("u", "up_proj"), ("d", "down_proj")):
            base = f"{pre}mlp.experts.{e}.{proj}.weight"
            recs.append((base + ".scale", np.asarray(L[nm + "s"][e], np.float32)))
            recs.append((base + "." + q, L[nm + "q"][e]))
    return recs
