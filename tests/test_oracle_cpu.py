"""CPU: the oracle restatement against the reference's golden vectors and,
where the reference compiled here (oracle/_ref), against the reference itself."""
import hashlib
import os

import numpy as np
import pytest

from helpers import GOLDEN, quant, small_layer, synth
from oracle.oracle import Port, Ref, quantize_q4, quantize_q8


@pytest.fixture(scope="module")
def port():
    return Port()


def test_quantizers_match_export_py(port):
    g = np.load(os.path.join(GOLDEN, "quant.npz"))
    s8, q8 = quantize_q8(g["W"])
    s4, q4 = quantize_q4(g["W"])
    assert np.array_equal(s8, g["s8"]) and np.array_equal(q8, g["q8"])
    assert np.array_equal(s4, g["s4"]) and np.array_equal(q4, g["q4"])
    # the C restatement too
    q, s = port.quantize(g["W"], 2)
    assert np.array_equal(q, g["q8"]) and np.array_equal(s, g["s8"])
    q, s = port.quantize(g["W"], 3)
    assert np.array_equal(q, g["q4"]) and np.array_equal(s, g["s4"])


def test_synth_stream_is_pinned():
    # first samples of the counter-based stream (guards the generator itself)
    a = synth(1, 4, 1.0)
    b = synth(1, 8, 1.0)
    assert np.array_equal(a, b[:4])
    assert np.all(np.isfinite(b)) and abs(float(synth(5, 100000, 1.0).std()) - 1.0) < 0.02


def test_oracle_synth_stream_equals_product_stream(port):
    # the benchmark's reference arm draws its inputs from the oracle's copy of
    # the stream; it must be the product's stream bit for bit
    import moe_cuda as mc
    for seed, off, n, std in ((1, 0, 4096, 1.0), (7000, 0, 2048 * 16, 1.0), (123456789, 77, 3000, 0.02)):
        assert np.array_equal(port.synth_normal(seed, n, std, off), mc.synth_normal_host(seed, n, std, off))


@pytest.mark.parametrize("dt", [2, 3])
def test_port_gemv_c1_matches_reference_golden(port, dt):
    g = np.load(os.path.join(GOLDEN, "gemv.npz"))
    W = synth(1, 768 * 2048, 0.02).reshape(768, 2048)
    x = synth(2, 2048, 1.0).reshape(1, 2048)
    s, q = quant(dt)(W)
    assert hashlib.sha256(q.tobytes() + s.tobytes()).digest() == g[f"c1_qsha_{dt}"].tobytes()
    y = port.matmul(x, q, s, 768, 2048, dt)[0]
    assert np.array_equal(y, g[f"c1_y_{dt}"])


@pytest.mark.parametrize("shape", [(3, 40, 96), (1, 17, 64), (5, 8, 2)])
@pytest.mark.parametrize("dt", [0, 2, 3])
def test_port_gemv_small_matches_reference_golden(port, shape, dt):
    M, N, K = shape
    g = np.load(os.path.join(GOLDEN, "gemv.npz"))
    Ws = synth(21 + K, N * K, 0.02).reshape(N, K)
    A = synth(22 + K, M * K, 1.0).reshape(M, K)
    if dt == 0:
        y = port.matmul(A, Ws, None, N, K, 0)
    else:
        s, q = quant(dt)(Ws)
        y = port.matmul(A, q, s, N, K, dt)
    assert np.array_equal(y, g[f"y_{M}_{N}_{K}_{dt}"])


@pytest.mark.parametrize("dt", [2, 3])
def test_port_moe_block_matches_reference_golden(port, dt):
    g = np.load(os.path.join(GOLDEN, "moe_small.npz"))
    L = small_layer(16, 256, 64, dt, bias=(dt == 3))
    xo, idx, p, lg = port.moe_block(g[f"xn_{dt}"], g[f"x_{dt}"], L)
    assert np.array_equal(lg, g[f"logits_{dt}"])
    assert np.array_equal(idx, g[f"idx_{dt}"])
    assert np.array_equal(p, g[f"p_{dt}"])
    assert np.array_equal(xo, g[f"xo_{dt}"])


@pytest.mark.skipif(not Ref.available(), reason="reference not compiled here (oracle/_ref)")
@pytest.mark.parametrize("dt", [2, 3])
def test_port_equals_reference_at_qwen_shape(port, dt):
    """Qwen3-30B-A3B shape (E=128, D=2048, F=768), T=2: the port's MoE block is
    bit-identical to the reference's layer_forward_f32 MoE block."""
    rng = np.random.default_rng(dt)
    E, D, F = 128, 2048, 768
    L = {"dtype": dt, "topk": 8,
         "router_w": (rng.standard_normal((E, D), np.float32) * 0.02),
         "router_b": rng.standard_normal(E).astype(np.float32) if dt == 3 else None}
    for nm, (r, c) in (("g", (F, D)), ("u", (F, D)), ("d", (D, F))):
        W = (rng.standard_normal((E * r, c), np.float32) * 0.02)
        s, q = quant(dt)(W)
        L[nm + "s"] = s.reshape(E, r)
        L[nm + "q"] = q.reshape(E, r, -1)
    x = rng.standard_normal((2, D), np.float32)
    ref = Ref()
    xo, xn, lg, idx, p = ref.moe_layer(x, L)
    xo2, idx2, p2, lg2 = port.moe_block(xn, x, L)
    assert np.array_equal(lg, lg2) and np.array_equal(idx, idx2)
    assert np.array_equal(p, p2) and np.array_equal(xo, xo2)


def test_port_rejects_odd_k_q4(port):
    with pytest.raises(AssertionError):
        port.matmul(np.zeros((1, 3), np.float32), np.zeros(4, np.uint8), np.ones(2, np.float32), 2, 3, 3)
