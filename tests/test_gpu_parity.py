"""GPU parity: libmoe_cuda (through its C-ABI) against the oracle and the
reference's golden vectors. Bar: bit-exact for quantisation and GEMV (integer
dots, IEEE-rounded epilogues); MoE layer outputs bit-exact as well (the
tolerance north_star allows, 1e-4·max|y|, is asserted first, then exact
equality), identical top-k."""
import os

import numpy as np
import pytest

from helpers import GOLDEN, layer_to_numpy, quant, small_layer, synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def port():
    from oracle.oracle import Port
    return Port()


def assert_moe_close(out, ref, idx, ref_idx):
    assert np.array_equal(idx, ref_idx), "top-k selection differs"
    tol = 1e-4 * float(np.abs(ref).max())
    err = float(np.abs(out - ref).max())
    assert err <= tol, f"max-abs {err} > 1e-4*max|y| = {tol}"


# ---- quantisers (export.py:23-36) -------------------------------------------

@pytest.mark.parametrize("dt", [2, 3])
def test_device_quantizer_bit_exact(gpu, dt):
    g = np.load(os.path.join(GOLDEN, "quant.npz"))
    for W in (g["W"], synth(1, 768 * 2048, 0.02).reshape(768, 2048)):
        Wd = torch.from_numpy(W).cuda()
        rows, cols = W.shape
        q = torch.empty(rows, cols if dt == 2 else cols // 2, dtype=torch.int8 if dt == 2 else torch.uint8,
                        device="cuda")
        s = torch.empty(rows, device="cuda")
        gpu.quantize_rowwise_dev(Wd, q, s, dt)
        torch.cuda.synchronize()
        s_ref, q_ref = quant(dt)(W)
        assert np.array_equal(q.cpu().numpy(), q_ref)
        assert np.array_equal(s.cpu().numpy(), s_ref)
    gq = g["q8"] if dt == 2 else g["q4"]
    assert np.array_equal(quant(dt)(g["W"])[1], gq)


# ---- matmul_f32_q8 / _q4 / matmul_adaptive (kernels.c) ----------------------

@pytest.mark.parametrize("dt", [2, 3])
def test_matmul_c1_matches_reference_golden(gpu, dt):
    g = np.load(os.path.join(GOLDEN, "gemv.npz"))
    W = synth(1, 768 * 2048, 0.02).reshape(768, 2048)
    x = synth(2, 2048, 1.0).reshape(1, 2048)
    s, q = quant(dt)(W)
    fn = gpu.matmul_f32_q8 if dt == 2 else gpu.matmul_f32_q4
    y = fn(x, q, s, 768, 2048)[0]
    assert np.array_equal(y, g[f"c1_y_{dt}"])
    qw = gpu.QuantizedWeight(q.ctypes.data, s.ctypes.data, 768, 2048, dt)
    assert np.array_equal(gpu.matmul_adaptive(x, None, qw, 768, 2048)[0], g[f"c1_y_{dt}"])


@pytest.mark.parametrize("shape", [(3, 40, 96), (1, 17, 64), (5, 8, 2)])
@pytest.mark.parametrize("dt", [0, 2, 3])
def test_matmul_ragged_shapes_match_reference_golden(gpu, shape, dt):
    M, N, K = shape
    g = np.load(os.path.join(GOLDEN, "gemv.npz"))
    Ws = synth(21 + K, N * K, 0.02).reshape(N, K)
    A = synth(22 + K, M * K, 1.0).reshape(M, K)
    if dt == 0:
        y = gpu.matmul_adaptive(A, Ws, None, N, K)
    else:
        s, q = quant(dt)(Ws)
        y = (gpu.matmul_f32_q8 if dt == 2 else gpu.matmul_f32_q4)(A, q, s, N, K)
    assert np.array_equal(y, g[f"y_{M}_{N}_{K}_{dt}"])


@pytest.mark.parametrize("dt", [2, 3])
@pytest.mark.parametrize("MNK", [(1, 2048, 768), (7, 768, 2048), (33, 256, 4096), (2, 100, 512)])
def test_matmul_fast_path_vs_port(gpu, port, dt, MNK):
    M, N, K = MNK
    W = synth(50 + K + N, N * K, 0.02).reshape(N, K)
    A = synth(51 + M, M * K, 1.5).reshape(M, K)
    s, q = quant(dt)(W)
    y = (gpu.matmul_f32_q8 if dt == 2 else gpu.matmul_f32_q4)(A, q, s, N, K)
    assert np.array_equal(y, port.matmul(A, q, s, N, K, dt))
    # device-pointer form
    Ad, qd, sd = (torch.from_numpy(a).cuda() for a in (A, q, s))
    Cd = torch.empty(M, N, device="cuda")
    gpu.matmul_q_dev(Ad, qd, sd, Cd, dt)
    gpu.check_status()
    assert np.array_equal(Cd.cpu().numpy(), y)


@pytest.mark.parametrize("dt", [2, 3])
def test_matmul_large_activations_stay_exact(gpu, port, dt):
    """|x| beyond the fast path's limb range (Q8 16 bits, Q4 8 bits): the exact
    fix-up pass recomputes on the device, for the host entry and for the
    device entry, as the reference computes it."""
    K, N = 512, 64
    W = synth(60, N * K, 0.02).reshape(N, K)
    A = synth(61, 2 * K, 1.0).reshape(2, K) * (400.0 if dt == 2 else 30.0)
    s, q = quant(dt)(W)
    want = port.matmul(A, q, s, N, K, dt)
    fn = gpu.matmul_f32_q8 if dt == 2 else gpu.matmul_f32_q4
    assert np.array_equal(fn(A, q, s, N, K), want)
    C = torch.empty(2, N, device="cuda")
    gpu.matmul_q_dev(torch.from_numpy(A).cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), C, dt)
    torch.cuda.synchronize()
    gpu.check_status()
    assert np.array_equal(C.cpu().numpy(), want)
    # the batched form, one row against two matrices
    qs = [torch.from_numpy(q).cuda(), torch.from_numpy(q[::-1].copy()).cuda()]
    ss = [torch.from_numpy(s).cuda(), torch.from_numpy(s[::-1].copy()).cuda()]
    qp = torch.tensor([t.data_ptr() for t in qs], dtype=torch.int64, device="cuda")
    sp = torch.tensor([t.data_ptr() for t in ss], dtype=torch.int64, device="cuda")
    Cb = torch.empty(2, N, device="cuda")
    xd = torch.from_numpy(A[:1].copy()).cuda()
    gpu.check(gpu.lib().moe_matmul_batched_dev(xd.data_ptr(), qp.data_ptr(), sp.data_ptr(), Cb.data_ptr(),
                                               2, N, K, dt, None))
    torch.cuda.synchronize()
    gpu.check_status()
    assert np.array_equal(Cb[0].cpu().numpy(), want[0])
    assert np.array_equal(Cb[1].cpu().numpy(), port.matmul(A[:1], q[::-1].copy(), s[::-1].copy(), N, K, dt)[0])


def test_matmul_adaptive_unknown_dtype_zero_fills(gpu):
    A = np.ones((2, 32), np.float32)
    qw = gpu.QuantizedWeight(None, None, 4, 32, 7)
    assert np.array_equal(gpu.matmul_adaptive(A, None, qw, 4, 32), np.zeros((2, 4), np.float32))


@pytest.mark.parametrize("dt", [2, 3])
def test_batched_gemv_matches_single(gpu, dt, port):
    n_mat, N, K = 6, 768, 2048
    x = synth(70, K, 1.0).reshape(1, K)
    qs, ss = [], []
    for i in range(n_mat):
        s, q = quant(dt)(synth(71 + i, N * K, 0.02).reshape(N, K))
        qs.append(torch.from_numpy(q).cuda()); ss.append(torch.from_numpy(s).cuda())
    qp = torch.tensor([t.data_ptr() for t in qs], dtype=torch.int64, device="cuda")
    sp = torch.tensor([t.data_ptr() for t in ss], dtype=torch.int64, device="cuda")
    C = torch.empty(n_mat, N, device="cuda")
    xd = torch.from_numpy(x).cuda()
    gpu.check(gpu.lib().moe_matmul_batched_dev(xd.data_ptr(), qp.data_ptr(), sp.data_ptr(),
                                               C.data_ptr(), n_mat, N, K, dt, None))
    gpu.check_status()
    for i in range(n_mat):
        ref = port.matmul(x, qs[i].cpu().numpy(), ss[i].cpu().numpy(), N, K, dt)[0]
        assert np.array_equal(C[i].cpu().numpy(), ref)


# ---- fused MoE block (test_model_trace.c:463-517) ----------------------------

@pytest.mark.parametrize("dt", [2, 3])
def test_moe_ffn_small_matches_reference_golden(gpu, dt):
    g = np.load(os.path.join(GOLDEN, "moe_small.npz"))
    L = small_layer(16, 256, 64, dt, bias=(dt == 3))
    gpu.upload_layer(100 + dt, L)
    xo, idx, p = gpu.moe_ffn_host(100 + dt, g[f"xn_{dt}"], g[f"x_{dt}"])
    assert np.array_equal(idx, g[f"idx_{dt}"])
    assert_moe_close(xo, g[f"xo_{dt}"], idx, g[f"idx_{dt}"])
    assert np.array_equal(xo, g[f"xo_{dt}"]), "not bit-exact (within tolerance)"
    assert np.array_equal(p, g[f"p_{dt}"])
    # the resident copy also serves the reference-shaped matmul entry points
    x1 = g[f"xn_{dt}"][:1]
    fn = gpu.matmul_f32_q8 if dt == 2 else gpu.matmul_f32_q4
    assert np.array_equal(fn(x1, L["gq"][3], L["gs"][3], 64, 256),
                          fn(x1, L["gq"][3].copy(), L["gs"][3].copy(), 64, 256))
    gpu.free_layer(100 + dt)


_QW = {}


def qwen_layer(gpu, dt, bias):
    key = (dt, bias)
    if key not in _QW:
        import synth as sy
        Ld = sy.make_layer_dev(torch, 1, 0, 128, 2048, 768, dt, bias=bias)
        torch.cuda.synchronize()
        lid = 200 + dt * 2 + int(bias)
        gpu.upload_layer(lid, Ld, device_arrays=True)
        gpu.check_status()
        _QW[key] = (lid, layer_to_numpy(Ld))
    return _QW[key]


@pytest.mark.parametrize("dt,T,bias", [(2, 1, False), (2, 4, False), (2, 16, False), (2, 32, True),
                                       (3, 1, False), (3, 16, False), (3, 512, True), (2, 100, True),
                                       (3, 2048, True), (2, 2048, True)])
def test_moe_ffn_qwen_shape_vs_port(gpu, port, dt, T, bias):
    lid, L = qwen_layer(gpu, dt, bias)
    xn = synth(900 + T, T * 2048, 1.0).reshape(T, 2048)
    xa = synth(901 + T, T * 2048, 1.0).reshape(T, 2048)
    ref, ref_idx, ref_p, _ = port.moe_block(xn, xa, L)
    xo, idx, p = gpu.moe_ffn_host(lid, xn, xa)
    assert_moe_close(xo, ref, idx, ref_idx)
    # bit-exact: integer dots, the reference's float order, and an expf equal
    # to the C library's (expf_ref.h)
    assert np.array_equal(xo, ref), f"only {float(np.mean(xo == ref)):.6f} of outputs bit-identical"
    assert np.array_equal(p, ref_p)


@pytest.mark.parametrize("dt,T", [(2, 1), (2, 16), (2, 40), (2, 100), (3, 1), (3, 16), (3, 64), (3, 300)])
def test_moe_ffn_tensor_core_path_equals_gemv_path(gpu, dt, T):
    """The tcgen05 grouped-GEMM path and the CUDA-core GEMV path compute the
    same integers, so their outputs are identical bit for bit (Q8: two
    activation limbs; Q4: nibbles unpacked in shared memory)."""
    lid, L = qwen_layer(gpu, dt, False)
    xn = torch.from_numpy(synth(960 + T, T * 2048, 1.0).reshape(T, 2048)).cuda()
    xa = torch.from_numpy(synth(961 + T, T * 2048, 1.0).reshape(T, 2048)).cuda()
    outs = []
    for flags in (gpu.FORCE_GEMM, gpu.FORCE_GEMV):
        o = xa.clone()
        gpu.moe_ffn_dev(lid, xn, o, flags=flags)
        torch.cuda.synchronize()
        gpu.check_status()
        outs.append(o.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])


def test_moe_ffn_device_ptrs_and_partial_combine(gpu, port):
    lid, L = qwen_layer(gpu, 2, False)
    T = 8
    xn = torch.from_numpy(synth(950, T * 2048, 1.0).reshape(T, 2048)).cuda()
    xa = torch.from_numpy(synth(951, T * 2048, 1.0).reshape(T, 2048)).cuda()
    out = xa.clone()
    idx = torch.empty(T, 8, dtype=torch.int32, device="cuda")
    p = torch.empty(T, 8, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        gpu.moe_ffn_dev(lid, xn, out, idx, p, stream=s)
    s.synchronize()
    gpu.check_status()
    ref, ref_idx, _, _ = port.moe_block(xn.cpu().numpy(), xa.cpu().numpy(), L)
    assert np.array_equal(out.cpu().numpy(), ref)
    # expert-parallel building blocks on a world of 1: partial + combine == moe_ffn
    y = torch.empty(T * 8, 2048, device="cuda")
    p2 = torch.empty(T, 8, device="cuda")
    gpu.moe_ffn_partial(lid, xn, y, None, p2)
    out2 = xa.clone()
    gpu.moe_ffn_combine(y, p2, out2)
    torch.cuda.synchronize()
    gpu.check_status()
    assert np.array_equal(out2.cpu().numpy(), ref)


def test_moe_ffn_empty_and_errors(gpu):
    lid, _ = qwen_layer(gpu, 2, False)
    x = np.zeros((0, 2048), np.float32)
    gpu.check(gpu.lib().moe_ffn(lid, x.ctypes.data, x.ctypes.data, 0, None, None, gpu.HOST_PTRS, None))
    with pytest.raises(gpu.MoeError):
        gpu.moe_ffn_host(9999, np.zeros((1, 2048), np.float32), np.zeros((1, 2048), np.float32))


# ---- .bin weight file straight into residency (model.h:212-305) -----------------

@pytest.mark.parametrize("dt", [2, 3])
def test_load_bin_layer_matches_reference_golden(gpu, dt, tmp_path):
    """The golden layer written as a .bin (the writer is pinned to export.py's
    bytes), loaded by moe_cuda_load_bin_layer: same output as the reference's
    layer_forward_f32, and as the same layer through moe_cuda_upload_layer."""
    from helpers import layer_records, write_bin
    g = np.load(os.path.join(GOLDEN, "moe_small.npz"))
    L = small_layer(16, 256, 64, dt, bias=(dt == 3))
    decoy = small_layer(16, 256, 64, dt, bias=False, seed_base=5)
    path = str(tmp_path / "w.bin")
    write_bin(path, layer_records(decoy, 6) + layer_records(L, 7) + layer_records(decoy, 8))
    assert gpu.bin_layer_info(path, 7) == (16, 256, 64, dt, int(dt == 3))
    gpu.load_bin_layer(path, 7, 200 + dt)
    xo, idx, p = gpu.moe_ffn_host(200 + dt, g[f"xn_{dt}"], g[f"x_{dt}"])
    assert np.array_equal(idx, g[f"idx_{dt}"])
    assert np.array_equal(xo, g[f"xo_{dt}"])
    assert np.array_equal(p, g[f"p_{dt}"])
    gpu.upload_layer(300 + dt, L)
    assert gpu.layer_bytes(200 + dt) == gpu.layer_bytes(300 + dt)
    x = synth(77, 24 * 256, 1.0).reshape(24, 256)
    xa = synth(78, 24 * 256, 1.0).reshape(24, 256)
    a = gpu.moe_ffn_host(200 + dt, x, xa)
    b = gpu.moe_ffn_host(300 + dt, x, xa)
    for u, v in zip(a, b):
        assert np.array_equal(u, v)
    gpu.free_layer(200 + dt)
    gpu.free_layer(300 + dt)


def test_load_bin_layer_errors(gpu):
    ref = os.path.join(GOLDEN, "layer_ref.bin")
    with pytest.raises(gpu.MoeError) as ei:
        gpu.load_bin_layer(ref, 0, 210)                  # no such layer in the file
    assert ei.value.code == gpu.MOE_ERR_INVALID
    with pytest.raises(gpu.MoeError) as ei:
        gpu.load_bin_layer(ref, 3, 210)                  # 3 experts (and Q4 rows of 8 bytes)
    assert ei.value.code == gpu.MOE_ERR_UNSUPPORTED
    with pytest.raises(gpu.MoeError) as ei:
        gpu.load_bin_layer(ref, 1, 211)                  # 3 experts: fewer than the top 8
    assert ei.value.code == gpu.MOE_ERR_UNSUPPORTED


@pytest.mark.parametrize("dt", [2, 3])
def test_load_bin_layer_qwen_shape(gpu, dt, tmp_path):
    """A Qwen3-shaped layer (D=2048, F=768, 32 experts) streamed from a .bin:
    resident bytes and moe_ffn outputs (tensor-core / fused paths, T=16 and
    T=96) identical to the same layer through moe_cuda_upload_layer."""
    import time
    from helpers import layer_records, write_bin
    L = small_layer(32, 2048, 768, dt, bias=True, seed_base=3)
    path = str(tmp_path / "q.bin")
    write_bin(path, layer_records(L, 0))
    t0 = time.perf_counter()
    gpu.load_bin_layer(path, 0, 220 + dt)
    dt_s = time.perf_counter() - t0
    print(f"load_bin_layer dtype {dt}: {os.path.getsize(path) / dt_s / 1e9:.2f} GB/s of file")
    gpu.upload_layer(320 + dt, L)
    assert gpu.layer_bytes(220 + dt) == gpu.layer_bytes(320 + dt)
    for T in (16, 96):
        x = synth(80 + T, T * 2048, 1.0).reshape(T, 2048)
        xa = synth(81 + T, T * 2048, 1.0).reshape(T, 2048)
        a = gpu.moe_ffn_host(220 + dt, x, xa)
        b = gpu.moe_ffn_host(320 + dt, x, xa)
        for u, v in zip(a, b):
            assert np.array_equal(u, v)
    gpu.free_layer(220 + dt)
    gpu.free_layer(320 + dt)


@pytest.mark.parametrize("dt,T", [(2, 16), (3, 64)])
def test_moe_ffn_unaligned_residual_stream(gpu, port, dt, T):
    """x_inout 4 bytes off a 16-byte boundary (a view into a larger buffer):
    the combine takes its scalar form, results unchanged."""
    lid, L = qwen_layer(gpu, dt, False)
    xn = synth(990 + T, T * 2048, 1.0).reshape(T, 2048)
    xa = synth(991 + T, T * 2048, 1.0).reshape(T, 2048)
    ref, ref_idx, _, _ = port.moe_block(xn, xa, L)
    buf = torch.zeros(T * 2048 + 1, device="cuda")
    out = buf[1:].view(T, 2048)
    out.copy_(torch.from_numpy(xa))
    gpu.moe_ffn_dev(lid, torch.from_numpy(xn).cuda(), out)
    torch.cuda.synchronize()
    gpu.check_status()
    assert np.array_equal(out.cpu().numpy(), ref)
