"""ctypes mirror of include/moe_host.h (the C host driver, libmoe_host.so).

The driver keeps borrowed weight pointers, so this wrapper holds a reference
to every array it passes until the model is freed."""
import ctypes as C
import os

import numpy as np

import moe_cuda as mc

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_host.so")

EXPORTS = (
    "mh_create", "mh_free", "mh_last_error", "mh_set_globals", "mh_set_layer",
    "mh_config_from_bin", "mh_load_bin", "mh_synth", "mh_pos", "mh_reset", "mh_fill_kv",
    "mh_step", "mh_generate", "mh_pick_greedy", "mh_embed", "mh_attention", "mh_moe",
    "mh_head", "mh_advance", "mh_timing", "mh_timing_reset", "mh_ep_setup", "mh_ep_connect",
)
# include/moe_model.h (model.c's call surface, served by the same library)
MODEL_EXPORTS = ("layer_forward_f32", "model_forward_f32", "moe_model_release")

LAYER_FIELDS = ("Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo", "q_norm", "k_norm", "rms1_w", "rms2_w")


class MhConfig(C.Structure):
    """MhConfig (QwenConfig, model.h:9-22, without causal / top_k)."""
    _fields_ = [(n, C.c_int) for n in ("d_model", "n_layers", "head_dim", "n_q", "n_kv", "d_ff",
                                       "n_experts", "vocab_size")] + \
               [("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class MhLayerWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in LAYER_FIELDS]


_lib = None


def lib():
    global _lib
    if _lib is None:
        mc.lib()                      # libmoe_cuda first (the driver links it)
        if not os.path.exists(LIB_PATH):
            raise mc.MoeError(mc.MOE_ERR_NOT_INIT, f"{LIB_PATH} is not built (make -C moe.cc_b200 host)")
        L = C.CDLL(LIB_PATH)
        vp, i, f, u64 = C.c_void_p, C.c_int, C.c_float, C.c_uint64
        sig = {
            "mh_create": ([vp, i, i, i], vp), "mh_free": ([vp], None), "mh_last_error": ([], C.c_char_p),
            "mh_set_globals": ([vp, vp, vp, vp], i), "mh_set_layer": ([vp, i, vp], i),
            "mh_config_from_bin": ([C.c_char_p, vp], i), "mh_load_bin": ([vp, C.c_char_p], i),
            "mh_synth": ([vp, u64, i, f], i), "mh_pos": ([vp], i), "mh_reset": ([vp], None),
            "mh_fill_kv": ([vp, i, u64, f], i), "mh_step": ([vp, vp, i, vp], i),
            "mh_generate": ([vp, vp, i, i, vp], i), "mh_pick_greedy": ([vp, vp, vp], i),
            "mh_embed": ([vp, vp, i, vp], i), "mh_attention": ([vp, i, vp, i, vp, vp], i),
            "mh_moe": ([vp, i, vp, vp, i], i), "mh_head": ([vp, vp, i, vp], i),
            "mh_advance": ([vp, i], i), "mh_timing": ([vp, vp, vp, vp], i),
            "mh_timing_reset": ([vp], None),
            "mh_ep_setup": ([vp, i, vp], i), "mh_ep_connect": ([vp, vp], i),
        }
        sig["layer_forward_f32"] = ([vp, i, i, vp, f] + [vp] * 10 + [i, i, i, i, f, vp, f, vp, vp] + [vp] * 6 +
                                    [i, i, i, vp, vp, vp, vp], None)
        sig["model_forward_f32"] = ([vp, i, vp, vp, i, vp], None)
        sig["moe_model_release"] = ([], None)
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes, fn.restype = args, res
        _lib = L
    return _lib


def check(rc):
    if rc != 0:
        raise mc.MoeError(rc, lib().mh_last_error().decode(errors="replace"))


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, np.float32)


def config_from_bin(path):
    c = MhConfig()
    check(lib().mh_config_from_bin(os.fsencode(path), C.byref(c)))
    return {n: getattr(c, n) for n, _ in MhConfig._fields_}


class HostModel:
    """One MhModel. cfg: dict with MhConfig's fields."""

    def __init__(self, cfg, batch=1, max_ctx=256, moe_base=0):
        self.cfg = dict(cfg)
        self.batch = batch
        c = MhConfig(**{n: cfg[n] for n, _ in MhConfig._fields_})
        self.h = lib().mh_create(C.byref(c), batch, max_ctx, moe_base)
        if not self.h:
            raise mc.MoeError(mc.MOE_ERR_INVALID, lib().mh_last_error().decode(errors="replace"))
        self._keep = []

    def close(self):
        if self.h:
            lib().mh_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _hold(self, a):
        a = _f32(a)
        if a is not None:
            self._keep.append(a)
            return a.ctypes.data
        return None

    def set_globals(self, tok_emb, final_norm_w, lm_head=None):
        check(lib().mh_set_globals(self.h, self._hold(tok_emb), self._hold(final_norm_w), self._hold(lm_head)))

    def set_layer(self, layer, w):
        lw = MhLayerWeights(**{n: self._hold(w.get(n)) for n in LAYER_FIELDS})
        check(lib().mh_set_layer(self.h, layer, C.byref(lw)))

    def pos(self):
        return lib().mh_pos(self.h)

    def reset(self):
        lib().mh_reset(self.h)

    def embed(self, ids):
        ids = np.ascontiguousarray(ids, np.int32).reshape(self.batch, -1)
        T = ids.shape[1]
        x = np.empty((self.batch * T, self.cfg["d_model"]), np.float32)
        check(lib().mh_embed(self.h, ids.ctypes.data, T, x.ctypes.data))
        return x

    def attention(self, layer, x, T):
        x = _f32(x)
        xa = np.empty_like(x)
        xn = np.empty_like(x)
        check(lib().mh_attention(self.h, layer, x.ctypes.data, T, xa.ctypes.data, xn.ctypes.data))
        return xa, xn

    def moe(self, layer, x_norm2, x_after, T):
        xa = np.array(x_after, np.float32, copy=True, order="C")
        xn = _f32(x_norm2)
        check(lib().mh_moe(self.h, layer, xn.ctypes.data, xa.ctypes.data, T))
        return xa

    def head(self, x, T):
        x = _f32(x)
        out = np.empty((self.batch, self.cfg["vocab_size"]), np.float32)
        check(lib().mh_head(self.h, x.ctypes.data, T, out.ctypes.data))
        return out

    def advance(self, T):
        check(lib().mh_advance(self.h, T))

    def step(self, ids):
        ids = np.ascontiguousarray(ids, np.int32).reshape(self.batch, -1)
        out = np.empty((self.batch, self.cfg["vocab_size"]), np.float32)
        check(lib().mh_step(self.h, ids.ctypes.data, ids.shape[1], out.ctypes.data))
        return out

    def generate(self, prompts, steps):
        prompts = np.ascontiguousarray(prompts, np.int32).reshape(self.batch, -1)
        out = np.empty((self.batch, steps), np.int32)
        check(lib().mh_generate(self.h, prompts.ctypes.data, prompts.shape[1], steps, out.ctypes.data))
        return out

    def pick_greedy(self, logits):
        lg = np.array(logits, np.float32, copy=True, order="C")
        ids = np.empty(self.batch, np.int32)
        check(lib().mh_pick_greedy(self.h, lg.ctypes.data, ids.ctypes.data))
        return ids

    def load_bin(self, path):
        check(lib().mh_load_bin(self.h, os.fsencode(path)))

    def synth(self, seed, expert_dtype, std=0.02):
        check(lib().mh_synth(self.h, seed, expert_dtype, std))

    def fill_kv(self, ctx, seed, std=1.0):
        check(lib().mh_fill_kv(self.h, ctx, seed, std))

    def timing(self):
        L = self.cfg["n_layers"]
        ms = np.zeros(L, np.float64)
        calls = np.zeros(L, np.int64)
        cpu = C.c_double(0)
        check(lib().mh_timing(self.h, ms.ctypes.data, calls.ctypes.data, C.byref(cpu)))
        return ms, calls, cpu.value


# ---- model.c's call surface (include/moe_model.h) ---------------------------

class QwenConfig(C.Structure):
    """model.h:9-22."""
    _fields_ = [(n, C.c_int) for n in ("d_model", "n_layers", "head_dim", "n_q", "n_kv", "d_ff", "n_experts",
                                       "top_k", "vocab_size", "causal")] + \
               [("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class QwenLayerWeights(C.Structure):
    """model.h:34-59."""
    _fields_ = [(n, C.c_void_p) for n in LAYER_FIELDS[:10]] + \
               [(n, C.c_void_p) for n in ("rms1_w", "rms2_w", "router_w", "router_b",
                                           "Wg", "bg", "Wu", "bu", "Wd", "bd", "Wg_q", "Wu_q", "Wd_q")] + \
               [("experts_quantized", C.c_int)]


class QwenWeights(C.Structure):
    """model.h:61-70."""
    _fields_ = [("tok_emb", C.c_void_p), ("final_norm_w", C.c_void_p), ("lm_head", C.c_void_p),
                ("layers", C.c_void_p)]


def _ptr_array(arrs):
    return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def model_forward_f32(ids, cfg, g, attn, moe_f32, apply_softmax=False):
    """model_forward_f32 (model.c:192-198) through libmoe_host.so: logits
    [T][vocab]. cfg: dict of QwenConfig fields; g: tok_emb, final_norm_w,
    lm_head (or None); attn: per layer LAYER_FIELDS dicts; moe_f32: per layer
    dicts router_w, router_b (or None), gate [E][F][D], up, down [E][D][F]."""
    keep = []

    def ptr(a):
        if a is None:
            return None
        a = np.ascontiguousarray(a, np.float32)
        keep.append(a)
        return a.ctypes.data
    L = cfg["n_layers"]
    layers = (QwenLayerWeights * L)()
    for l in range(L):
        lw = layers[l]
        for n in LAYER_FIELDS:
            setattr(lw, n, ptr(attn[l].get(n)))
        lw.router_w = ptr(moe_f32[l]["router_w"])
        lw.router_b = ptr(moe_f32[l].get("router_b"))
        for n, key in (("Wg", "gate"), ("Wu", "up"), ("Wd", "down")):
            a = np.ascontiguousarray(moe_f32[l][key], np.float32)
            keep.append(a)
            arr = _ptr_array([a[e] for e in range(a.shape[0])])
            keep.append(arr)
            setattr(lw, n, C.addressof(arr))
    keep.append(layers)
    w = QwenWeights(ptr(g["tok_emb"]), ptr(g["final_norm_w"]), ptr(g.get("lm_head")), C.addressof(layers))
    c = QwenConfig(**{k: cfg[k] for k, _ in QwenConfig._fields_})
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.empty((len(ids), cfg["vocab_size"]), np.float32)
    lib().model_forward_f32(ids.ctypes.data, len(ids), C.byref(c), C.byref(w), int(apply_softmax), out.ctypes.data)
    return out


def layer_forward_f32(x, a, rms1_eps, rms2_eps, n_q, n_kv, head_dim, causal, rope_theta, router_w, router_b,
                      gate, up, down, top_k, reuse=None):
    """layer_forward_f32 (model.c:38-58) on one layer, x [T][D] updated and
    returned. a: LAYER_FIELDS dict; gate/up [E][F][D], down [E][D][F] fp32;
    reuse: optional (idx [T][top_k] int32, p [T][top_k]) routing."""
    x = np.array(x, np.float32, copy=True, order="C")
    T, D = x.shape
    keep = []

    def ptr(v):
        if v is None:
            return None
        v = np.ascontiguousarray(v, np.float32)
        keep.append(v)
        return v.ctypes.data
    E, F = gate.shape[0], gate.shape[1]
    arrs = []
    for m in (gate, up, down):
        m = np.ascontiguousarray(m, np.float32)
        keep.append(m)
        arrs.append(_ptr_array([m[e] for e in range(E)]))
    Dq, Dkv = n_q * head_dim, n_kv * head_dim
    scratch = np.zeros(T * (Dq + 2 * Dkv) + T * T + T * Dq + 2 * T * D, np.float32)
    ri = rp = None
    if reuse is not None:
        ri = np.ascontiguousarray(reuse[0], np.int32)
        rp = np.ascontiguousarray(reuse[1], np.float32)
    lib().layer_forward_f32(x.ctypes.data, T, D, ptr(a["rms1_w"]), rms1_eps, ptr(a["Wq"]), ptr(a.get("bq")),
                            ptr(a["Wk"]), ptr(a.get("bk")), ptr(a["Wv"]), ptr(a.get("bv")), ptr(a["Wo"]),
                            ptr(a.get("bo")), ptr(a.get("q_norm")), ptr(a.get("k_norm")), n_q, n_kv, head_dim,
                            causal, rope_theta, ptr(a["rms2_w"]), rms2_eps, ptr(router_w), ptr(router_b),
                            C.addressof(arrs[0]), None, C.addressof(arrs[1]), None, C.addressof(arrs[2]), None,
                            E, top_k, F, scratch.ctypes.data, None,
                            None if ri is None else ri.ctypes.data, None if rp is None else rp.ctypes.data)
    return x


def model_release():
    lib().moe_model_release()
