"""GPU: model.c's call surface (include/moe_model.h, served by libmoe_host.so)
against the reference's own model.c, compiled from its source into
oracle/_ref (oracle/ref_shim.c). layer_forward_f32 (model.c:38-190) and
model_forward_f32 (model.c:192-252) run attention on the CPU and the fp32
experts' MoE block on the GPU; results must equal the reference's bit for
bit."""
import numpy as np
import pytest

from helpers import TINY, synth, tiny_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    from oracle.oracle import Ref
    if not Ref.available():
        pytest.skip("oracle/_ref (the reference compiled from its sources) is not built")
    return Ref()


@pytest.fixture(scope="module")
def mh(gpu):
    import moe_host
    yield moe_host
    moe_host.model_release()


def f32_experts(seed, E, D, F, std=0.3, bias=False):
    n = lambda k, shape, s: synth(seed + k, int(np.prod(shape)), s).reshape(shape)
    return {"router_w": n(0, (E, D), 0.5), "router_b": n(1, (E,), 0.5) if bias else None,
            "gate": n(2, (E, F, D), std), "up": n(3, (E, F, D), std), "down": n(4, (E, D, F), std)}


def tiny_f32(seed, top_k=8, bias=False):
    g, attn, _ = tiny_model(2, seed=seed, attn_bias=bias)
    c = TINY
    moe = [f32_experts(7000 + 50 * l + 10 * seed, c["n_experts"], c["d_model"], c["d_ff"], bias=bias)
           for l in range(c["n_layers"])]
    cfg = dict(c, top_k=top_k, causal=1, rms_eps=1e-6)
    return cfg, g, attn, moe


@pytest.mark.parametrize("top_k,softmax,bias", [(8, False, False), (2, True, True), (3, False, True)])
def test_model_forward_f32_matches_reference_model_c(mh, ref, top_k, softmax, bias):
    cfg, g, attn, moe = tiny_f32(1, top_k, bias)
    rng = np.random.default_rng(5 + top_k)
    for T in (1, 7, 12):
        ids = rng.integers(0, cfg["vocab_size"], T).astype(np.int32)
        want = ref.mc_model_forward(ids, cfg, g, attn, moe, apply_softmax=softmax)
        got = mh.model_forward_f32(ids, cfg, g, attn, moe, apply_softmax=softmax)
        mh.model_release()     # resident copies are keyed by host pointers, which numpy reuses
        assert got.shape == (T, cfg["vocab_size"])
        assert np.array_equal(got, want), f"T={T}: max-abs {np.abs(got - want).max()}"


@pytest.mark.parametrize("causal,qk_norm,reuse", [(1, True, False), (0, True, False), (1, False, True)])
def test_layer_forward_f32_matches_reference_model_c(mh, ref, causal, qk_norm, reuse):
    _, attn, _ = tiny_model(2, seed=3, attn_bias=True, qk_norm=qk_norm)
    a = attn[0]
    c = TINY
    m = f32_experts(7700, c["n_experts"], c["d_model"], c["d_ff"], bias=True)
    T = 9
    x = synth(7800, T * c["d_model"], 1.0).reshape(T, c["d_model"])
    routing = None
    if reuse:
        rng = np.random.default_rng(3)
        idx = np.stack([rng.permutation(c["n_experts"])[:4] for _ in range(T)]).astype(np.int32)
        p = rng.random((T, 4)).astype(np.float32)
        routing = (idx, p)
    top_k = 4 if reuse else 8
    args = (x, a, 1e-5, 2e-6, c["n_q"], c["n_kv"], c["head_dim"], causal, 1e4,
            m["router_w"], m["router_b"], m["gate"], m["up"], m["down"], top_k)
    want = ref.mc_layer_forward(*args, reuse=routing)
    got = mh.layer_forward_f32(*args, reuse=routing)
    mh.model_release()
    assert np.array_equal(got, want), f"max-abs {np.abs(got - want).max()}"


def test_layer_forward_f32_qwen_width(mh, ref):
    """Qwen3 widths for the MoE block (D=2048, F=768, top-8 of 16 experts)."""
    D, F, E, T = 2048, 768, 16, 3
    a = {"Wq": synth(7900, 128 * D, 0.02).reshape(128, D), "Wk": synth(7901, 64 * D, 0.02).reshape(64, D),
         "Wv": synth(7902, 64 * D, 0.02).reshape(64, D), "Wo": synth(7903, D * 128, 0.02).reshape(D, 128),
         "rms1_w": synth(7904, D, 0.1) + 1.0, "rms2_w": synth(7905, D, 0.1) + 1.0,
         "q_norm": synth(7906, 64, 0.1) + 1.0, "k_norm": synth(7907, 64, 0.1) + 1.0}
    m = f32_experts(7910, E, D, F, std=0.02)
    x = synth(7920, T * D, 1.0).reshape(T, D)
    args = (x, a, 1e-6, 1e-6, 2, 1, 64, 1, 1e6, m["router_w"], None, m["gate"], m["up"], m["down"], 8)
    want = ref.mc_layer_forward(*args)
    got = mh.layer_forward_f32(*args)
    mh.model_release()
    assert np.array_equal(got, want), f"max-abs {np.abs(got - want).max()}"
