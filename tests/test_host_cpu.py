"""The C host driver (include/moe_host.h) on the CPU: its KV-cached attention
and head, composed with the oracle's MoE block, against the reference's own
model_forward_f32 (test_model_trace.c:526-596, compiled from source into
oracle/_ref), which recomputes the whole prefix at every step. Bar: logits
bit for bit at every prefill and decode step."""
import numpy as np
import pytest

import moe_cuda as mc
from helpers import TINY, tiny_model

mh = pytest.importorskip("moe_host")
from oracle.oracle import Port, Ref  # noqa: E402

needs_ref = pytest.mark.skipif(not Ref.available(), reason="oracle/_ref (the reference's own code) not built")


def load(model, g, attn):
    model.set_globals(g["tok_emb"], g["final_norm_w"], g["lm_head"])
    for l, a in enumerate(attn):
        model.set_layer(l, a)


def cpu_step(model, port, moe, ids):
    """One driver step with the MoE block from the oracle instead of the GPU."""
    ids = np.asarray(ids, np.int32).reshape(model.batch, -1)
    T = ids.shape[1]
    x = model.embed(ids)
    for l in range(TINY["n_layers"]):
        xa, xn = model.attention(l, x, T)
        x = port.moe_block(xn, xa, moe[l])[0]
    logits = model.head(x, T)
    model.advance(T)
    return logits


@needs_ref
@pytest.mark.parametrize("dt,variant", [(2, {}), (3, {}), (2, {"attn_bias": True, "tied": True}),
                                        (3, {"qk_norm": False, "router_bias": True})])
def test_cached_decode_matches_reference_full_recompute(dt, variant):
    g, attn, moe = tiny_model(dt, seed=1, **variant)
    ref, port = Ref(), Port()
    B, P, steps = 2, 6, 5
    rng = np.random.default_rng(dt)
    seqs = [list(rng.integers(0, TINY["vocab_size"], P)) for _ in range(B)]
    model = mh.HostModel(TINY, batch=B, max_ctx=32)
    load(model, g, attn)
    logits = cpu_step(model, port, moe, np.array(seqs))
    for s in range(steps):
        for b in range(B):
            want = ref.model_forward(seqs[b], TINY, g, attn, moe)
            assert np.array_equal(logits[b], want), f"step {s} sequence {b}"
        nxt = model.pick_greedy(logits)
        for b in range(B):
            seqs[b].append(int(nxt[b]))
        logits = cpu_step(model, port, moe, nxt)
    assert model.pos() == P + steps


@needs_ref
def test_chunked_prefill_matches():
    """Prompt fed in chunks of 3, 1 and 4 tokens: same logits as one pass."""
    g, attn, moe = tiny_model(2, seed=2)
    ref, port = Ref(), Port()
    ids = list(np.random.default_rng(9).integers(0, TINY["vocab_size"], 8))
    model = mh.HostModel(TINY, batch=1, max_ctx=16)
    load(model, g, attn)
    pos = 0
    for n in (3, 1, 4):
        logits = cpu_step(model, port, moe, ids[pos:pos + n])
        pos += n
        assert np.array_equal(logits[0], ref.model_forward(ids[:pos], TINY, g, attn, moe))


def test_pick_greedy_first_maximum():
    model = mh.HostModel(TINY, batch=2, max_ctx=4)
    lg = np.zeros((2, TINY["vocab_size"]), np.float32)
    lg[0, 5] = lg[0, 9] = 3.0
    lg[1, -1] = 1.0
    assert list(model.pick_greedy(lg)) == [5, TINY["vocab_size"] - 1]


def test_errors_without_gpu_or_weights():
    model = mh.HostModel(TINY, batch=1, max_ctx=4)
    with pytest.raises(mc.MoeError):
        model.embed([1])                       # no embedding set
    g, attn, moe = tiny_model(2)
    load(model, g, attn)
    with pytest.raises(mc.MoeError):
        model.embed([TINY["vocab_size"]])      # id out of range
    x = model.embed([1])
    with pytest.raises(mc.MoeError):
        model.attention(0, np.vstack([x] * 5), 5)   # past max_ctx
    xa, xn = model.attention(0, x, 1)
    with pytest.raises(mc.MoeError):
        model.moe(0, xn, xa, 1)                # the MoE block needs the GPU library initialised
    bad = dict(TINY, n_q=3)
    with pytest.raises(mc.MoeError):
        mh.HostModel(bad)                      # n_q not a multiple of n_kv


def test_config_from_bin(tmp_path):
    from helpers import model_records, write_bin
    g, attn, moe = tiny_model(3, seed=1)
    p = str(tmp_path / "m.bin")
    write_bin(p, model_records(g, attn, moe))
    got = mh.config_from_bin(p)
    assert got == {k: (float(np.float32(v)) if isinstance(v, float) else v) for k, v in TINY.items()}
    # without q_norm the head size is inferred as rows/32 (model.h:113-115)
    g2, attn2, moe2 = tiny_model(3, seed=1, qk_norm=False)
    write_bin(p, model_records(g2, attn2, moe2))
    assert mh.config_from_bin(p)["head_dim"] == TINY["n_q"] * TINY["head_dim"] // 32


@pytest.mark.parametrize("D", [60, 64, 72])
def test_head_is_the_reference_chain(D):
    """mh_head = rmsnorm_forward_f32 then matmul_f32 (test_model_trace.c:213-255),
    restated as scalar float32 loops, for row lengths with and without a
    remainder of 8 (the vector path's tail)."""
    cfg = dict(TINY, d_model=D, vocab_size=37)
    rng = np.random.default_rng(D)
    emb = rng.standard_normal((37, D), dtype=np.float32)
    head = rng.standard_normal((37, D), dtype=np.float32)
    fn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    x = rng.standard_normal((1, D), dtype=np.float32)
    model = mh.HostModel(cfg, batch=1, max_ctx=4)
    model.set_globals(emb, fn, head)
    got = model.head(x, 1)[0]
    f = np.float32
    msq = f(0)
    for v in x[0]:
        msq = f(msq + f(v * v))
    msq = f(msq / f(D))
    inv = f(f(1) / f(np.sqrt(f(msq + f(TINY["rms_eps"])))))
    y = [f(f(v * inv) * w) for v, w in zip(x[0], fn)]
    want = np.empty(37, np.float32)
    for n in range(37):
        acc = f(0)
        for k in range(D):
            acc = f(acc + f(y[k] * head[n, k]))
        want[n] = acc
    assert np.array_equal(got, want)


def test_scalar_path_too():
    """The portable matmul path (MOE_HOST_SCALAR=1, read once per process)."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, MOE_HOST_SCALAR="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", __file__,
                        "-k", "head_is or cached_decode or long_prefix"], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:]


def test_generate_program_fails_loudly_without_gpu():
    """moe_generate needs the GPU for the MoE block: without one it exits
    non-zero with the library's message, and runs no CPU substitute."""
    import os
    import subprocess
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    tool = os.path.join(os.path.dirname(mh.LIB_PATH), "moe_generate")
    r = subprocess.run([tool, "--layers", "1", "--steps", "2", "--prompt", "2"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode != 0 and "moe_cuda_init" in r.stderr and not r.stdout


@needs_ref
def test_long_prefix_matches_reference():
    """A 21-token prompt then decode to 27 positions: key blocks of 16 plus
    remainders in the attention scores, against the full recompute."""
    g, attn, moe = tiny_model(2, seed=3)
    ref, port = Ref(), Port()
    B = 2
    rng = np.random.default_rng(77)
    seqs = [list(rng.integers(0, TINY["vocab_size"], 21)) for _ in range(B)]
    model = mh.HostModel(TINY, batch=B, max_ctx=40)
    load(model, g, attn)
    logits = cpu_step(model, port, moe, np.array(seqs))
    for s in range(6):
        for b in range(B):
            assert np.array_equal(logits[b], ref.model_forward(seqs[b], TINY, g, attn, moe)), f"step {s}"
        nxt = model.pick_greedy(logits)
        for b in range(B):
            seqs[b].append(int(nxt[b]))
        logits = cpu_step(model, port, moe, nxt)
