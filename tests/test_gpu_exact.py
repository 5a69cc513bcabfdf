"""GPU parity for activations outside the fast kernels' integer range.

The reference truncates every activation with no range limit, (int32_t)(a*127)
for Q8 and (int32_t)(a*7) for Q4 (kernels.c:66, :113), and accumulates in
int32. The fast kernels carry 16-bit (Q8) or 8-bit (Q4) activations; a token
whose x, or the h of one of its slots, leaves that range is recomputed by the
exact fix-up pass (exact.cu). These tests check that moe_ffn then returns
what the oracle (the reference's arithmetic) returns, on every path: the
routing kernel + two tcgen05 GEMMs (T=1), the fused kernel (T=16), the
prefill path (T=512), the CUDA-core GEMV path, device pointers, and
moe_ffn_partial. Also the routing edge cases of topk_desc
(test_model_trace.c:275-288): exact ties, NaN logits, all logits -inf."""
import numpy as np
import pytest

from helpers import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def port():
    from oracle.oracle import Port
    return Port()


_QW = {}


def qwen_layer(gpu, dt, bias=False):
    key = (dt, bias)
    if key not in _QW:
        import synth as sy
        from helpers import layer_to_numpy
        Ld = sy.make_layer_dev(torch, 1, 0, 128, 2048, 768, dt, bias=bias)
        torch.cuda.synchronize()
        lid = 300 + dt * 2 + int(bias)
        gpu.upload_layer(lid, Ld, device_arrays=True)
        gpu.check_status()
        _QW[key] = (lid, layer_to_numpy(Ld))
    return _QW[key]


def assert_matches(out, ref, idx, ref_idx, min_same=1.0):
    """Identical top-k, max-abs <= 1e-4 max|ref| over finite values (the
    north_star bar, asserted first for a readable failure), NaN where the
    reference has NaN, and every output bit-identical."""
    assert np.array_equal(idx, ref_idx), "top-k selection differs"
    assert np.array_equal(np.isnan(out), np.isnan(ref)), "NaN pattern differs"
    fin = np.isfinite(ref)
    tol = 1e-4 * float(np.abs(ref[fin]).max()) if fin.any() else 0.0
    err = float(np.abs(out[fin] - ref[fin]).max()) if fin.any() else 0.0
    assert err <= tol, f"max-abs {err} > 1e-4*max|y| = {tol}"
    same = float(np.mean((out == ref) | (np.isnan(out) & np.isnan(ref))))
    assert same >= min_same, f"only {same:.6f} of outputs bit-identical"


def q8_big(T, seed):
    """N(0,1) tokens; every third token (and token 0) gets elements up to
    |x| = 1000, beyond the 16-bit limbs (|x| < 258)."""
    x = synth(seed, T * 2048, 1.0).reshape(T, 2048)
    for t in range(0, T, 3):
        x[t, (t * 37) % 2048::97] *= 1000.0 / 4.0
        x[t, (t * 11) % 2048] = 1000.0 if t % 2 == 0 else -1000.0
    return x


def q4_big(T, seed, kind):
    """kind 'x': tokens with elements beyond |x| = 18.3 (trunc(7x) leaves s8);
    kind 'h': |x| <= 18 everywhere, but large enough that h = silu(g)*u leaves
    s8 in some slots (only h is out of range)."""
    x = synth(seed, T * 2048, 1.0).reshape(T, 2048)
    if kind == "x":
        for t in range(0, T, 3):
            x[t, (t * 13) % 2048::61] *= 30.0
            x[t, (t * 7) % 2048] = -40.0
    else:
        x = np.clip(x * 9.0, -18.0, 18.0).astype(np.float32)
    return x


@pytest.mark.parametrize("T", [1, 16, 512])
def test_q8_large_activations_host_ptrs(gpu, port, T):
    lid, L = qwen_layer(gpu, 2)
    xn = q8_big(T, 4100 + T)
    xa = synth(4200 + T, T * 2048, 1.0).reshape(T, 2048)
    assert np.abs(xn).max() >= 999.0
    ref, ref_idx, _, _ = port.moe_block(xn, xa, L)
    xo, idx, _ = gpu.moe_ffn_host(lid, xn, xa)
    assert_matches(xo, ref, idx, ref_idx)
    # the marks were cleared: an in-range call right after is unaffected
    xn2 = synth(4300 + T, T * 2048, 1.0).reshape(T, 2048)
    ref2, ref_idx2, _, _ = port.moe_block(xn2, xa, L)
    xo2, idx2, _ = gpu.moe_ffn_host(lid, xn2, xa)
    assert_matches(xo2, ref2, idx2, ref_idx2)


@pytest.mark.parametrize("T,kind", [(1, "x"), (16, "x"), (512, "x"), (1, "h"), (16, "h"), (512, "h")])
def test_q4_large_activations(gpu, port, T, kind):
    lid, L = qwen_layer(gpu, 3, bias=(T == 512))
    xn = q4_big(T, 4400 + T, kind)
    xa = synth(4500 + T, T * 2048, 1.0).reshape(T, 2048)
    if kind == "h":
        assert np.abs(xn).max() <= 18.0
    ref, ref_idx, _, _ = port.moe_block(xn, xa, L)
    xo, idx, _ = gpu.moe_ffn_host(lid, xn, xa)
    assert_matches(xo, ref, idx, ref_idx)


@pytest.mark.parametrize("dt,T", [(2, 16), (3, 16), (2, 100), (3, 64)])
def test_large_activations_gemv_path_and_device_ptrs(gpu, port, dt, T):
    """The CUDA-core GEMV path (forced) and the tensor-core path on device
    pointers, both with out-of-range tokens."""
    lid, L = qwen_layer(gpu, dt)
    xn_h = q8_big(T, 4600 + T) if dt == 2 else q4_big(T, 4600 + T, "x")
    xa_h = synth(4700 + T, T * 2048, 1.0).reshape(T, 2048)
    ref, ref_idx, _, _ = port.moe_block(xn_h, xa_h, L)
    xn = torch.from_numpy(xn_h).cuda()
    for flags in (gpu.FORCE_GEMM, gpu.FORCE_GEMV):
        out = torch.from_numpy(xa_h).cuda()
        idx = torch.empty(T, 8, dtype=torch.int32, device="cuda")
        gpu.moe_ffn_dev(lid, xn, out, idx, None, flags=flags)
        torch.cuda.synchronize()
        gpu.check_status()            # no MOE_ERR_RANGE: the fix-up computed them
        assert_matches(out.cpu().numpy(), ref, idx.cpu().numpy(), ref_idx)


def test_large_activations_partial_combine(gpu, port):
    lid, L = qwen_layer(gpu, 2)
    T = 8
    xn_h = q8_big(T, 4800)
    xa_h = synth(4801, T * 2048, 1.0).reshape(T, 2048)
    ref, ref_idx, _, _ = port.moe_block(xn_h, xa_h, L)
    xn = torch.from_numpy(xn_h).cuda()
    y = torch.empty(T * 8, 2048, device="cuda")
    p = torch.empty(T, 8, device="cuda")
    idx = torch.empty(T, 8, dtype=torch.int32, device="cuda")
    gpu.moe_ffn_partial(lid, xn, y, idx, p)
    out = torch.from_numpy(xa_h).cuda()
    gpu.moe_ffn_combine(y, p, out)
    torch.cuda.synchronize()
    gpu.check_status()
    assert_matches(out.cpu().numpy(), ref, idx.cpu().numpy(), ref_idx)


def test_constant_300_input(gpu, port):
    """x = 300 everywhere: trunc(127*300) needs 17 bits; the reference computes
    it, so the library does too (this call used to return MOE_ERR_RANGE)."""
    lid, L = qwen_layer(gpu, 2)
    xn = np.full((1, 2048), 300.0, np.float32)
    xa = np.zeros((1, 2048), np.float32)
    ref, ref_idx, _, _ = port.moe_block(xn, xa, L)
    xo, idx, _ = gpu.moe_ffn_host(lid, xn, xa)
    assert_matches(xo, ref, idx, ref_idx)


def test_nan_and_inf_activations(gpu, port):
    """NaN and +-inf in x: the reference's truncation gives INT32_MIN
    (x86 cvttss2si) and its router logits are NaN for that token, so no expert
    is chosen and p is NaN: the token's output is NaN. Other tokens are
    unaffected."""
    lid, L = qwen_layer(gpu, 2)
    T = 4
    xn = synth(4900, T * 2048, 1.0).reshape(T, 2048)
    xa = synth(4901, T * 2048, 1.0).reshape(T, 2048)
    xn[1, 5] = np.nan
    xn[2, 7] = np.inf
    ref, ref_idx, _, _ = port.moe_block(xn, xa, L)
    xo, idx, _ = gpu.moe_ffn_host(lid, xn, xa)
    assert np.isnan(ref[1]).all() and np.isnan(ref[2]).all() and np.isfinite(ref[0]).all()
    assert_matches(xo, ref, idx, ref_idx)


# ---- routing edge cases: topk_desc (test_model_trace.c:275-288) ---------------

def edge_layer(gpu, dt, lid, mutate):
    """The Qwen-shaped layer with a modified router (host copy), uploaded
    under its own id."""
    _, L = qwen_layer(gpu, dt)
    L2 = dict(L)
    L2["router_w"] = L["router_w"].copy()
    L2["router_b"] = None if L.get("router_b") is None else L["router_b"].copy()
    mutate(L2)
    gpu.upload_layer(lid, L2)
    return L2


@pytest.mark.parametrize("dt", [2, 3])
def test_router_exact_ties_pick_lower_index(gpu, port, dt):
    """Duplicate router rows give bit-equal logits; topk_desc's strict '>'
    keeps the lower expert index first. Rows 10, 40, 41, 90, 127 equal row 3."""
    def mutate(L):
        for e in (10, 40, 41, 90, 127):
            L["router_w"][e] = L["router_w"][3]
    L = edge_layer(gpu, dt, 390 + dt, mutate)
    T = 16
    xn = synth(5000, T * 2048, 1.0).reshape(T, 2048)
    # make expert 3's row win for several tokens: x along router row 3
    for t in range(0, T, 2):
        xn[t] += 0.5 * L["router_w"][3] / np.linalg.norm(L["router_w"][3]) * 40
    xa = synth(5001, T * 2048, 1.0).reshape(T, 2048)
    ref, ref_idx, _, logits = port.moe_block(xn, xa, L)
    assert any(list(r[:6]) == [3, 10, 40, 41, 90, 127] for r in ref_idx), "no tie was exercised"
    xo, idx, _ = gpu.moe_ffn_host(390 + dt, xn, xa)
    assert_matches(xo, ref, idx, ref_idx)
    gpu.free_layer(390 + dt)


def test_router_nan_logits_never_chosen(gpu, port):
    """A NaN router weight makes that expert's logit NaN for every token:
    never selected (v > val is false for NaN)."""
    def mutate(L):
        L["router_w"][5, 100] = np.nan
        L["router_w"][77, 0] = np.nan
    L = edge_layer(gpu, 2, 395, mutate)
    T = 16
    xn = synth(5100, T * 2048, 1.0).reshape(T, 2048)
    xa = synth(5101, T * 2048, 1.0).reshape(T, 2048)
    ref, ref_idx, _, logits = port.moe_block(xn, xa, L)
    assert np.isnan(logits[:, 5]).all() and not np.isin(ref_idx, [5, 77]).any()
    xo, idx, _ = gpu.moe_ffn_host(395, xn, xa)
    assert_matches(xo, ref, idx, ref_idx)
    gpu.free_layer(395)


def test_router_all_minus_inf(gpu, port):
    """A router bias of -inf on every expert: no logit exceeds -inf, so
    topk_desc keeps idx -1 and the softmax gives p = NaN (exp(-inf - -inf));
    the reference's output for the token is then NaN (p * y). With -inf on all
    but 5 experts, the 3 empty slots have p = 0 and add nothing."""
    def mutate(L):
        b = np.full(128, -np.inf, np.float32)
        L["router_b"] = b
    L = edge_layer(gpu, 2, 396, mutate)
    T = 2
    xn = synth(5200, T * 2048, 1.0).reshape(T, 2048)
    xa = synth(5201, T * 2048, 1.0).reshape(T, 2048)
    ref, ref_idx, _, _ = port.moe_block(xn, xa, L)
    assert (ref_idx == -1).all() and np.isnan(ref).all()
    xo, idx, _ = gpu.moe_ffn_host(396, xn, xa)
    assert_matches(xo, ref, idx, ref_idx)
    gpu.free_layer(396)

    def mutate5(L):
        b = np.full(128, -np.inf, np.float32)
        b[[2, 9, 50, 51, 120]] = 0.0
        L["router_b"] = b
    L = edge_layer(gpu, 2, 397, mutate5)
    ref, ref_idx, _, _ = port.moe_block(xn, xa, L)
    assert (ref_idx[:, 5:] == -1).all() and np.isfinite(ref).all()
    xo, idx, _ = gpu.moe_ffn_host(397, xn, xa)
    assert_matches(xo, ref, idx, ref_idx)
    gpu.free_layer(397)
