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
            a = np.require(a, requirements="C")   # keeps 0-d arrays 0-d
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


# ---- a tiny full model (host driver tests) -----------------------------------
TINY = dict(d_model=64, n_layers=2, head_dim=16, n_q=4, n_kv=2, d_ff=32, n_experts=8,
            vocab_size=97, rope_theta=1e7, rms_eps=1e-6)   # theta and eps of model.h:119-120


def tiny_model(dt, seed=0, attn_bias=False, qk_norm=True, tied=False, router_bias=False, expert_std=0.3):
    """Seeded weights of a TINY-shaped Qwen3-MoE model: globals (tok_emb,
    final_norm_w, lm_head or None), per-layer attention dicts (MhLayerWeights
    field names) and per-layer MoE dicts in the upload layout. With
    expert_std 0.3 the down projection's inputs reach trunc(7h) of several
    hundred, beyond the fast Q4 kernels' 8-bit range, so the GPU runs use the
    exact fix-up pass."""
    c = TINY
    D, hd, nq, nkv, E, F, V = (c[k] for k in ("d_model", "head_dim", "n_q", "n_kv", "n_experts",
                                              "d_ff", "vocab_size"))
    s = 5000 + 100 * seed

    def n(k, shape, std, mean=0.0):
        return (synth(s + k, int(np.prod(shape)), std).reshape(shape) + np.float32(mean)).astype(np.float32)

    g = {"tok_emb": n(0, (V, D), 1.0), "final_norm_w": n(1, (D,), 0.1, 1.0),
         "lm_head": None if tied else n(2, (V, D), 0.1)}
    attn, moe = [], []
    for l in range(c["n_layers"]):
        b = 10 + 40 * l
        a = {"Wq": n(b, (nq * hd, D), 0.15), "Wk": n(b + 1, (nkv * hd, D), 0.15),
             "Wv": n(b + 2, (nkv * hd, D), 0.15), "Wo": n(b + 3, (D, nq * hd), 0.1),
             "rms1_w": n(b + 4, (D,), 0.1, 1.0), "rms2_w": n(b + 5, (D,), 0.1, 1.0)}
        if qk_norm:
            a["q_norm"] = n(b + 6, (hd,), 0.1, 1.0)
            a["k_norm"] = n(b + 7, (hd,), 0.1, 1.0)
        if attn_bias:
            a["bq"], a["bk"] = n(b + 8, (nq * hd,), 0.1), n(b + 9, (nkv * hd,), 0.1)
            a["bv"], a["bo"] = n(b + 10, (nkv * hd,), 0.1), n(b + 11, (D,), 0.1)
        attn.append(a)
        L = {"dtype": dt, "topk": 8, "router_w": n(b + 12, (E, D), 0.5),
             "router_b": n(b + 13, (E,), 0.5) if router_bias else None}
        for j, (nm, rows, cols) in enumerate((("g", F, D), ("u", F, D), ("d", D, F))):
            ss, qs = [], []
            for e in range(E):
                sc, q = quant(dt)(n(b + 14 + 3 * e + j, (rows, cols), expert_std))
                ss.append(sc); qs.append(q)
            L[nm + "s"] = np.ascontiguousarray(np.stack(ss))
            L[nm + "q"] = np.ascontiguousarray(np.stack(qs))
        moe.append(L)
    return g, attn, moe


def model_records(g, attn, moe):
    """A whole tiny model as .bin records, with the tensor names the reference's
    loader reads (model.h:162-210)."""
    recs = [("model.embed_tokens.weight", g["tok_emb"]), ("model.norm.weight", g["final_norm_w"])]
    if g.get("lm_head") is not None:
        recs.append(("lm_head.weight", g["lm_head"]))
    names = {"Wq": "self_attn.q_proj.weight", "Wk": "self_attn.k_proj.weight", "Wv": "self_attn.v_proj.weight",
             "Wo": "self_attn.o_proj.weight", "bq": "self_attn.q_proj.bias", "bk": "self_attn.k_proj.bias",
             "bv": "self_attn.v_proj.bias", "bo": "self_attn.o_proj.bias", "q_norm": "self_attn.q_norm.weight",
             "k_norm": "self_attn.k_norm.weight", "rms1_w": "input_layernorm.weight",
             "rms2_w": "post_attention_layernorm.weight"}
    for l, a in enumerate(attn):
        for k, nm in names.items():
            if a.get(k) is not None:
                recs.append((f"model.layers.{l}.{nm}", a[k]))
        recs += layer_records(moe[l], l)
    return recs
