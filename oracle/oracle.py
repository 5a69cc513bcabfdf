"""CPU oracle for the MoE expert-FFN path — TEST INFRASTRUCTURE ONLY.

Loaded only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, always as the checker (never as the thing measured or shipped).

* ``Port``: ctypes binding of oracle/liboracle.so, this repo's C restatement
  (oracle/moe_oracle.c) of kernels.c:51-181 and test_model_trace.c:213-288,
  463-517, and of export.py:23-36.
* ``Ref``: ctypes binding of oracle/_ref/libmoe_ref.so, the reference's own
  kernels.c + test_model_trace.c compiled from their sources (oracle/Makefile);
  present wherever the reference sources were present at build time.
* ``quantize_q8``/``quantize_q4``: numpy restatement of export._rowwise_q8/_q4
  (export.py:23-36), pinned bit-exact against the reference's torch code by
  tests/golden/make_golden.py.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmoe_ref.so")

_f = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def build():
    """Build liboracle.so (and _ref when the reference sources exist)."""
    import subprocess
    subprocess.check_call(["make", "-s", "-C", HERE])


class Port:
    def __init__(self, path=PORT_SO):
        if not os.path.exists(path):
            build()
        self.lib = C.CDLL(path)
        vp, i = C.c_void_p, C.c_int
        for name in ("orc_matmul_q8", "orc_matmul_q4"):
            getattr(self.lib, name).argtypes = [vp, vp, vp, vp, i, i, i]
            getattr(self.lib, name).restype = i
        self.lib.orc_matmul_f32.argtypes = [vp, vp, vp, i, i, i]
        self.lib.orc_moe_block.argtypes = [vp, vp, vp, i, i, i, i, i, vp, vp, i,
                                           vp, vp, vp, vp, vp, vp, vp, vp, vp]
        self.lib.orc_moe_block.restype = i
        self.lib.orc_quantize_q8.argtypes = [vp, i, i, vp, vp]
        self.lib.orc_quantize_q4.argtypes = [vp, i, i, vp, vp]
        self.lib.orc_quantize_q4.restype = i
        self.lib.orc_synth_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_size_t, C.c_float, vp]

    def matmul(self, A, q, s, N, K, dtype):
        A = np.ascontiguousarray(A, np.float32)
        M = A.shape[0]
        out = np.empty((M, N), np.float32)
        if dtype == 2:
            r = self.lib.orc_matmul_q8(_p(A), _p(q), _p(s), _p(out), M, N, K)
        elif dtype == 3:
            r = self.lib.orc_matmul_q4(_p(A), _p(q), _p(s), _p(out), M, N, K)
        else:
            self.lib.orc_matmul_f32(_p(A), _p(q), _p(out), M, N, K)
            r = 0
        assert r == 0
        return out

    def moe_block(self, x_norm2, x_after, L):
        """L: dict with router_w, router_b (or None), dtype, gq, gs, uq, us, dq, ds, topk."""
        T, D = x_norm2.shape
        E = L["router_w"].shape[0]
        F = L["gs"].shape[1]
        topk = L.get("topk", 8)
        out = np.empty((T, D), np.float32)
        idx = np.empty((T, topk), np.int32)
        p = np.empty((T, topk), np.float32)
        logits = np.empty((T, E), np.float32)
        r = self.lib.orc_moe_block(
            _p(x_norm2), _p(x_after), _p(out), T, D, E, topk, F,
            _p(L["router_w"]), _p(L.get("router_b")), L["dtype"],
            _p(L["gq"]), _p(L["gs"]), _p(L["uq"]), _p(L["us"]), _p(L["dq"]), _p(L["ds"]),
            _p(idx), _p(p), _p(logits))
        assert r == 0
        return out, idx, p, logits

    def synth_normal(self, seed, n, std, offset=0):
        """n values of the seeded N(0, std) stream (benchmark inputs)."""
        out = np.empty(n, np.float32)
        self.lib.orc_synth_normal(seed & ((1 << 64) - 1), offset, n, std, _p(out))
        return out

    def quantize(self, W, dtype):
        W = np.ascontiguousarray(W, np.float32)
        rows, cols = W.shape
        s = np.empty(rows, np.float32)
        if dtype == 2:
            q = np.empty((rows, cols), np.int8)
            self.lib.orc_quantize_q8(_p(W), rows, cols, _p(q), _p(s))
        else:
            q = np.empty((rows, cols // 2), np.uint8)
            assert self.lib.orc_quantize_q4(_p(W), rows, cols, _p(q), _p(s)) == 0
        return q, s


class Ref:
    """The reference's own compiled C (oracle/_ref)."""

    @staticmethod
    def available():
        return os.path.exists(REF_SO)

    def __init__(self, path=REF_SO):
        self.lib = C.CDLL(path)
        vp, i = C.c_void_p, C.c_int
        self.lib.ref_moe_layer.argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, i, i,
                                           vp, vp, i, vp, vp, vp, vp, vp, vp]
        self.lib.ref_moe_layer.restype = i
        self.lib.ref_matmul.argtypes = [vp, vp, vp, vp, vp, i, i, i, i]

    def model_forward(self, ids, cfg, g, attn, moe):
        """The reference's model_forward_f32 (test_model_trace.c:526-596):
        logits of the last of ids. cfg: TINY-style dict; g/attn/moe as built
        by tests/helpers.tiny_model."""
        names = ("Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo", "q_norm", "k_norm", "rms1_w", "rms2_w")
        keep = []

        def ptr(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a)
            keep.append(a)
            return a.ctypes.data
        L = cfg["n_layers"]
        ap = (C.c_void_p * (12 * L))(*[ptr(attn[l].get(n)) for l in range(L) for n in names])
        rp = (C.c_void_p * (2 * L))(*[ptr(moe[l][k]) for l in range(L) for k in ("router_w", "router_b")])
        ep = (C.c_void_p * (6 * L))(*[ptr(moe[l][k]) for l in range(L)
                                      for k in ("gq", "gs", "uq", "us", "dq", "ds")])
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(cfg["vocab_size"], np.float32)
        f = self.lib.ref_model_forward
        f.argtypes = [C.c_void_p] + [C.c_int] * 9 + [C.c_float] * 2 + [C.c_void_p] * 5 + [C.c_int, C.c_void_p,
                                                                                           C.c_void_p]
        f.restype = C.c_int
        r = f(ids.ctypes.data, len(ids), cfg["d_model"], L, cfg["head_dim"], cfg["n_q"], cfg["n_kv"],
              cfg["d_ff"], cfg["n_experts"], cfg["vocab_size"], cfg["rope_theta"], cfg["rms_eps"],
              ptr(g["tok_emb"]), ptr(g["final_norm_w"]), ptr(g.get("lm_head")), ap, rp, moe[0]["dtype"], ep,
              out.ctypes.data)
        assert r == 0
        return out

    def mc_model_forward(self, ids, cfg, g, attn, moe_f32, apply_softmax=False):
        """model.c's model_forward_f32 (model.c:192-252, compiled from its
        source by oracle/ref_shim.c): logits of every row [T][vocab].
        moe_f32: per layer dicts router_w, router_b, gate, up, down (fp32)."""
        names = ("Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo", "q_norm", "k_norm", "rms1_w", "rms2_w")
        keep = []

        def ptr(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return a.ctypes.data
        L = cfg["n_layers"]
        ap = (C.c_void_p * (12 * L))(*[ptr(attn[l].get(n)) for l in range(L) for n in names])
        rp = (C.c_void_p * (2 * L))(*[ptr(moe_f32[l][k]) if moe_f32[l].get(k) is not None else None
                                      for l in range(L) for k in ("router_w", "router_b")])
        ep = (C.c_void_p * (3 * L))(*[ptr(moe_f32[l][k]) for l in range(L) for k in ("gate", "up", "down")])
        ids = np.ascontiguousarray(ids, np.int32)
        T = len(ids)
        out = np.empty((T, cfg["vocab_size"]), np.float32)
        f = self.lib.ref_mc_model_forward
        f.argtypes = [C.c_void_p] + [C.c_int] * 10 + [C.c_float, C.c_int] + [C.c_void_p] * 6 + [C.c_int, C.c_void_p]
        f.restype = C.c_int
        F, E = moe_f32[0]["gate"].shape[1], moe_f32[0]["gate"].shape[0]
        r = f(ids.ctypes.data, T, cfg["d_model"], L, cfg["head_dim"], cfg["n_q"], cfg["n_kv"], F, E,
              cfg["top_k"], cfg["vocab_size"], cfg["rope_theta"], cfg["causal"],
              ptr(g["tok_emb"]), ptr(g["final_norm_w"]), ptr(g.get("lm_head")), ap, rp, ep,
              int(apply_softmax), out.ctypes.data)
        assert r == 0
        return out

    def mc_layer_forward(self, x, a, rms1_eps, rms2_eps, n_q, n_kv, head_dim, causal, rope_theta,
                         router_w, router_b, gate, up, down, top_k, reuse=None):
        """model.c's layer_forward_f32 (model.c:38-190) on one layer: x after it."""
        names = ("Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo", "q_norm", "k_norm", "rms1_w", "rms2_w")
        keep = []

        def ptr(v):
            if v is None:
                return None
            v = np.ascontiguousarray(v, np.float32)
            keep.append(v)
            return v.ctypes.data
        x = np.array(x, np.float32, copy=True, order="C")
        T, D = x.shape
        E, F = gate.shape[0], gate.shape[1]
        ap = (C.c_void_p * 12)(*[ptr(a.get(n)) for n in names])
        ri = rp = None
        if reuse is not None:
            ri = np.ascontiguousarray(reuse[0], np.int32)
            rp = np.ascontiguousarray(reuse[1], np.float32)
        f = self.lib.ref_mc_layer_forward
        f.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_float, C.c_float, C.c_int, C.c_int, C.c_int,
                      C.c_int, C.c_float] + [C.c_void_p] * 5 + [C.c_int] * 3 + [C.c_void_p] * 2
        f.restype = C.c_int
        r = f(x.ctypes.data, T, D, ap, rms1_eps, rms2_eps, n_q, n_kv, head_dim, causal, rope_theta,
              ptr(router_w), ptr(router_b), ptr(gate), ptr(up), ptr(down), E, top_k, F,
              None if ri is None else ri.ctypes.data, None if rp is None else rp.ctypes.data)
        assert r == 0
        return x

    def matmul(self, A, q, s, N, K, dtype):
        A = np.ascontiguousarray(A, np.float32)
        M = A.shape[0]
        out = np.empty((M, N), np.float32)
        if dtype == 0:
            self.lib.ref_matmul(_p(A), None, None, _p(q), _p(out), M, N, K, 0)
        else:
            self.lib.ref_matmul(_p(A), _p(q), _p(s), None, _p(out), M, N, K, dtype)
        return out

    def moe_layer(self, x, L):
        """Run the reference's layer_forward_f32 (zero attention). Returns
        x_out, x_norm2 (the MoE input), logits, idx, p."""
        x = np.ascontiguousarray(x, np.float32)
        T, D = x.shape
        E = L["router_w"].shape[0]
        F = L["gs"].shape[1]
        topk = L.get("topk", 8)
        out = np.empty((T, D), np.float32)
        xn = np.empty((T, D), np.float32)
        logits = np.empty((T, E), np.float32)
        idx = np.empty((T, topk), np.int32)
        p = np.empty((T, topk), np.float32)
        r = self.lib.ref_moe_layer(
            _p(x), _p(out), _p(xn), _p(logits), _p(idx), _p(p), T, D, E, topk, F,
            _p(L["router_w"]), _p(L.get("router_b")), L["dtype"],
            _p(L["gq"]), _p(L["gs"]), _p(L["uq"]), _p(L["us"]), _p(L["dq"]), _p(L["ds"]))
        assert r == 0
        return out, xn, logits, idx, p


def quantize_q8(w):
    """export._rowwise_q8 (export.py:23-27) restated in numpy."""
    w = np.ascontiguousarray(w, np.float32)
    s = np.maximum(np.abs(w).max(axis=1, keepdims=True), np.float32(1e-8)) / np.float32(127.0)
    s = s.astype(np.float32)
    q = np.rint(w / s).astype(np.int8)
    return s[:, 0].copy(), q


def quantize_q4(w):
    """export._rowwise_q4 (export.py:29-36) restated in numpy."""
    w = np.ascontiguousarray(w, np.float32)
    s = (np.maximum(np.abs(w).max(axis=1, keepdims=True), np.float32(1e-8)) / np.float32(7.0)).astype(np.float32)
    q = np.clip(np.rint(w / s), -8, 7).astype(np.int8)
    q = (q + 8).astype(np.uint8)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return s[:, 0].copy(), np.ascontiguousarray(packed)
