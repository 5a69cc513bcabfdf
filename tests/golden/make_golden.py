"""Generate tests/golden/*.npz from the REFERENCE itself.

Run where the reference sources are present (a checkout named `reference`
beside this repository's, or the directory MOE_REF_DIR names) after
`make -C oracle`:

    python tests/golden/make_golden.py

* quant.npz  — export._rowwise_q8 / _rowwise_q4 (export.py:23-36), imported
  from the reference and run on seeded and hand-made edge-case rows.
* gemv.npz   — the reference's matmul_adaptive (kernels.c:149-181, compiled
  from source into oracle/_ref) on config C1 (768x2048, Q8 and Q4) and on
  small ragged shapes.
* moe_small.npz — the reference's layer_forward_f32 MoE block
  (test_model_trace.c:463-517, via oracle/ref_shim.c) on a small seeded layer.
* host_tiny.npz — the reference's model_forward_f32 (test_model_trace.c:526-596)
  on tests/helpers.tiny_model weights (Q8 and Q4), two sequences: a 6-token
  prompt then greedy decode, the logits of every step, recomputed over the
  whole prefix as the reference does. `python tests/golden/make_golden.py
  host` writes only this file.
* mkbin_ref.bin — a tiny random-init model (2 layers, D=64, 8 experts, Q4)
  dumped per tensor as export.py --outdir does (export._save_tensor,
  export._rowwise_q4, export.py:130-178) and merged by the reference's own
  merge_dir.py. moe_mkbin must write these bytes for the same arguments.
  `python tests/golden/make_golden.py mkbin` writes only this file.
* layer_ref.bin — a tiny weight file written by the reference's own writer
  (export.MAGIC, export._save_tensor, export._rowwise_q8/_q4): two MoE
  layers (Q8 at index 1, Q4 with a router bias at index 3, router under the
  mlp.router.gate.weight name), a norm weight and a repeated name. Pins the
  tests' .bin writer (byte for byte) and the loader's parse.
  `python tests/golden/make_golden.py bin` writes only this file.

Inputs come from the counter-based normal stream moe_synth_normal_host of
libmoe_cuda.so (host code, no GPU needed), so tests can rebuild them.
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "moe.cc_b200"))
# the reference checkout, by default beside this repository's checkout
REF_DIR = os.environ.get("MOE_REF_DIR", os.path.join(os.path.dirname(ROOT), "reference"))
OUT = os.path.dirname(os.path.abspath(__file__))


def synth(seed, n, std):
    import moe_cuda as mc
    return mc.synth_normal_host(seed, n, std)


def edge_rows():
    """Rows that hit round-half-even ties, the 1e-8 clamp and the Q4 clamp."""
    r0 = np.zeros(64, np.float32)                                  # all-zero row
    r1 = np.array([127.0] + [k + 0.5 for k in range(-31, 32)], np.float32)  # s=1 ties (Q8)
    r2 = np.array([7.0] + [((k % 15) - 7) + 0.5 for k in range(63)], np.float32)  # s=1 ties (Q4)
    r3 = np.full(64, 1e-12, np.float32)                            # below the clamp
    r4 = np.linspace(-3.0, 3.0, 64).astype(np.float32)
    return np.stack([r0, r1, r2, r3, r4])


def main():
    sys.path.insert(0, REF_DIR)
    import torch
    import export  # the reference's exporter (its quantisers)
    if sys.argv[1:] == ["mkbin"]:
        mkbin_fixture(torch, export)
        return
    if sys.argv[1:] == ["host"]:
        host_fixture()
        print("host_tiny.npz written to", OUT)
        return
    bin_fixture(torch, export)
    if sys.argv[1:] == ["bin"]:
        print("layer_ref.bin written to", OUT)
        return
    from oracle.oracle import Ref

    ref = Ref()
    # ---- quantisers ----
    Wq = np.concatenate([synth(11, 8 * 64, 0.02).reshape(8, 64), edge_rows()])
    s8, q8 = export._rowwise_q8(torch.from_numpy(Wq))
    s4, q4 = export._rowwise_q4(torch.from_numpy(Wq))
    np.savez(os.path.join(OUT, "quant.npz"), W=Wq, s8=s8.numpy(), q8=q8.numpy(),
             s4=s4.numpy(), q4=q4.numpy())

    # ---- GEMV: config C1 + small ragged shapes ----
    g = {}
    W = synth(1, 768 * 2048, 0.02).reshape(768, 2048)
    x = synth(2, 2048, 1.0).reshape(1, 2048)
    for dt, fn in ((2, export._rowwise_q8), (3, export._rowwise_q4)):
        s, q = fn(torch.from_numpy(W))
        s, q = s.numpy(), q.numpy()
        g[f"c1_y_{dt}"] = ref.matmul(x, q, s, 768, 2048, dt)[0]
        g[f"c1_qsha_{dt}"] = np.frombuffer(hashlib.sha256(q.tobytes() + s.tobytes()).digest(), np.uint8)
    for (M, N, K) in ((3, 40, 96), (1, 17, 64), (5, 8, 2)):
        Ws = synth(21 + K, N * K, 0.02).reshape(N, K)
        A = synth(22 + K, M * K, 1.0).reshape(M, K)
        for dt, fn in ((2, export._rowwise_q8), (3, export._rowwise_q4)):
            s, q = fn(torch.from_numpy(Ws))
            g[f"y_{M}_{N}_{K}_{dt}"] = ref.matmul(A, q.numpy(), s.numpy(), N, K, dt)
        g[f"y_{M}_{N}_{K}_0"] = ref.matmul(A, Ws, None, N, K, 0)
    np.savez(os.path.join(OUT, "gemv.npz"), **g)

    # ---- small MoE layer through the reference's layer_forward_f32 ----
    m = {}
    E, D, F, T = 16, 256, 64, 5
    for dt, fn, bias in ((2, export._rowwise_q8, False), (3, export._rowwise_q4, True)):
        L = small_layer(E, D, F, dt, bias, fn, torch)
        xin = synth(40 + dt, T * D, 1.0).reshape(T, D)
        xo, xn, lg, idx, p = ref.moe_layer(xin, L)
        m.update({f"x_{dt}": xin, f"xo_{dt}": xo, f"xn_{dt}": xn, f"logits_{dt}": lg,
                  f"idx_{dt}": idx, f"p_{dt}": p})
    np.savez(os.path.join(OUT, "moe_small.npz"), **m)
    print("golden fixtures written to", OUT)


def bin_fixture(torch, export):
    """layer_ref.bin through the reference's writer (export.py:188-206)."""
    import struct
    recs = [("model.norm.weight", torch.from_numpy(synth(60, 32, 1.0)))]
    for layer, dt, fn, bias, rname in ((1, 2, export._rowwise_q8, False, "mlp.gate.weight"),
                                        (3, 3, export._rowwise_q4, True, "mlp.router.gate.weight")):
        E, D, F = 3, 32, 16
        pre = f"model.layers.{layer}."
        recs.append((pre + rname, torch.from_numpy(synth(61 + layer, E * D, 0.02).reshape(E, D))))
        if bias:
            recs.append((pre + "mlp.gate.bias", torch.from_numpy(synth(62 + layer, E, 1.0))))
        q = "q8" if dt == 2 else "q4"
        for e in range(E):
            for j, (proj, rows, cols) in enumerate((("gate_proj", F, D), ("up_proj", F, D),
                                                    ("down_proj", D, F))):
                w = torch.from_numpy(synth(700 + 10 * layer + 3 * e + j, rows * cols, 0.02).reshape(rows, cols))
                s, qq = fn(w)
                base = f"{pre}mlp.experts.{e}.{proj}.weight"
                recs += [(base + ".scale", s), (base + "." + q, qq)]
    # a repeated name: the reader keeps the first record (io.c:333-338)
    recs.append(("model.norm.weight", torch.zeros(32)))
    with open(os.path.join(OUT, "layer_ref.bin"), "wb") as f:
        f.write(export.MAGIC)
        f.write(struct.pack("<I", len(recs)))
        for name, t in recs:
            export._save_tensor(f, name, t)


MKBIN_ARGS = dict(layers=2, d_model=64, n_q=4, n_kv=2, head_dim=16, d_ff=32, experts=8, vocab=97,
                  seed=3, quant="q4")


def mkbin_fixture(torch, export):
    """mkbin_ref.bin: export --outdir layout merged by merge_dir.py."""
    import json
    import shutil
    import struct
    import tempfile
    a = MKBIN_ARGS
    D, hd, nq, nkv, F, E, V = (a[k] for k in ("d_model", "head_dim", "n_q", "n_kv", "d_ff", "experts", "vocab"))

    def t(layer, tid, shape):
        sd = (a["seed"] * 1000003 + layer * 1009 + tid) & ((1 << 64) - 1)
        return torch.from_numpy(synth(sd, int(np.prod(shape)), 0.02).reshape(shape))
    tensors = [("model.embed_tokens.weight", t(65535, 0, (V, D)))]
    for L in range(a["layers"]):
        pre = f"model.layers.{L}."
        for j, (nm, shp) in enumerate((("q_proj", (nq * hd, D)), ("k_proj", (nkv * hd, D)),
                                        ("v_proj", (nkv * hd, D)), ("o_proj", (D, nq * hd)))):
            tensors.append((pre + f"self_attn.{nm}.weight", t(L, 100000 + j, shp)))
        tensors.append((pre + "self_attn.q_norm.weight", t(L, 100004, (hd,))))
        tensors.append((pre + "self_attn.k_norm.weight", t(L, 100005, (hd,))))
        tensors.append((pre + "mlp.gate.weight", t(L, 0, (E, D))))
        for e in range(E):
            for j, (nm, shp) in enumerate((("gate_proj", (F, D)), ("up_proj", (F, D)), ("down_proj", (D, F)))):
                tensors.append((pre + f"mlp.experts.{e}.{nm}.weight", t(L, 2 + 3 * e + j, shp)))
        tensors.append((pre + "input_layernorm.weight", t(L, 100006, (D,))))
        tensors.append((pre + "post_attention_layernorm.weight", t(L, 100007, (D,))))
    tensors.append(("model.norm.weight", t(65535, 1, (D,))))
    tensors.append(("lm_head.weight", t(65535, 2, (V, D))))
    tmp = tempfile.mkdtemp()
    try:
        manifest = {"tensors": []}
        for name, w in tensors:
            fn = export._sanitize(name) + ".bin"
            with open(os.path.join(tmp, fn), "wb") as f:      # export.py:143-170
                f.write(export.MAGIC)
                f.write(struct.pack("<I", 1))
                if export._is_expert_weight(name) and w.dim() == 2:
                    sc, q = export._rowwise_q4(w)
                    export._save_tensor(f, name + ".scale", sc)
                    export._save_tensor(f, name + ".q4", q)
                else:
                    export._save_tensor(f, name, w.float())
            manifest["tensors"].append({"name": name, "file": fn})
        with open(os.path.join(tmp, "manifest.json"), "w") as f:
            json.dump(manifest, f)
        import merge_dir                                        # the reference's merger
        argv = sys.argv
        sys.argv = ["merge_dir.py", os.path.join(OUT, "mkbin_ref.bin"), tmp]
        try:
            merge_dir.main()
        finally:
            sys.argv = argv
    finally:
        shutil.rmtree(tmp)


def host_fixture():
    """host_tiny.npz: greedy decode of two sequences through the reference."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from helpers import TINY, tiny_model
    from oracle.oracle import Ref
    ref = Ref()
    out = {}
    B, P, steps = 2, 6, 6
    for dt in (2, 3):
        g, attn, moe = tiny_model(dt, seed=1)
        rng = np.random.default_rng(100 + dt)
        seqs = [list(map(int, rng.integers(0, TINY["vocab_size"], P))) for _ in range(B)]
        out[f"prompt_{dt}"] = np.array(seqs, np.int32)
        logits = np.empty((steps, B, TINY["vocab_size"]), np.float32)
        for s in range(steps):
            for b in range(B):
                lg = ref.model_forward(seqs[b], TINY, g, attn, moe)
                logits[s, b] = lg
                # greedy: the first maximum of softmax(logits) (test_model_trace.c:723-731);
                # with the top two logits this far apart it is the logits' argmax
                top = np.sort(lg)[-2:]
                assert top[1] - top[0] > 1e-3
                seqs[b].append(int(np.argmax(lg)))
        out[f"logits_{dt}"] = logits
        out[f"tokens_{dt}"] = np.array([sq[P:] for sq in seqs], np.int32)
    np.savez(os.path.join(OUT, "host_tiny.npz"), **out)


def small_layer(E, D, F, dt, bias, quant, torch=None):
    """Seeded small layer; `quant` maps a [rows, cols] float32 array to (s, q)."""
    L = {"dtype": dt, "topk": 8,
         "router_w": synth(30 + dt, E * D, 0.02).reshape(E, D)}
    L["router_b"] = synth(31 + dt, E, 1.0) if bias else None
    shapes = {"g": (F, D), "u": (F, D), "d": (D, F)}
    for j, nm in enumerate("gud"):
        rows, cols = shapes[nm]
        ss, qs = [], []
        for e in range(E):
            w = synth(1000 * dt + 3 * e + j, rows * cols, 0.02).reshape(rows, cols)
            s, q = quant(torch.from_numpy(w) if torch is not None else w)
            ss.append(np.asarray(s)); qs.append(np.asarray(q))
        L[nm + "s"] = np.ascontiguousarray(np.stack(ss))
        L[nm + "q"] = np.ascontiguousarray(np.stack(qs))
    return L


if __name__ == "__main__":
    main()
