"""GPU: the allocation-free matmul entry point (moe_matmul_q_dev_noalloc).

It serves callers that may not allocate GPU memory when they call in (for
example code running inside an allocator or memory-pool callback, or a host
whose device memory is entirely reserved up front). It keeps its scratch in a
fixed array inside the library, so it must give exactly what the regular
entry points give, also on back-to-back calls that reuse that array.
Collected last on purpose (file name) so a stop-at-first-failure run has
already run everything else.
"""
import numpy as np
import pytest

from helpers import quant, synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def noalloc(mc, A, q, s, C, dt):
    M, K = A.shape
    N = C.shape[1]
    mc.check(mc.lib().moe_matmul_q_dev_noalloc(A.data_ptr(), q.data_ptr(), s.data_ptr(), C.data_ptr(),
                                               M, N, K, dt, None))


@pytest.mark.parametrize("dt", [2, 3])
def test_noalloc_matches_existing_entry_on_two_calls(gpu, dt):
    N, K = 768, 2048
    W = synth(300 + dt, N * K, 0.02).reshape(N, K)
    s, q = quant(dt)(W)
    qd, sd = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    # call 1: ordinary activations, against the regular device entry point
    A1 = synth(310 + dt, 5 * K, 1.0).reshape(5, K)
    A1d = torch.from_numpy(A1).cuda()
    ref1 = torch.empty(5, N, device="cuda")
    gpu.matmul_q_dev(A1d, qd, sd, ref1, dt)
    got1 = torch.empty(5, N, device="cuda")
    noalloc(gpu, A1d, qd, sd, got1, dt)
    torch.cuda.synchronize()
    gpu.check_status()
    assert np.array_equal(got1.cpu().numpy(), ref1.cpu().numpy())
    # call 2 reuses the same scratch: different rows, some activations far
    # outside the fast path's integer range, against the exact host entry
    A2 = synth(320 + dt, 3 * K, 1.0).reshape(3, K)
    A2[1, ::7] *= 500.0
    A2d = torch.from_numpy(A2).cuda()
    got2 = torch.empty(3, N, device="cuda")
    noalloc(gpu, A2d, qd, sd, got2, dt)
    torch.cuda.synchronize()
    fn = gpu.matmul_f32_q8 if dt == 2 else gpu.matmul_f32_q4
    assert np.array_equal(got2.cpu().numpy(), fn(A2, q, s, N, K))


@pytest.mark.parametrize("dt", [2, 3])
def test_noalloc_warmed_call_allocates_nothing(gpu, dt):
    """After the first call on the device (the set-up, which may load the
    library's kernels), a call leaves the device's free memory unchanged."""
    N, K = 512, 1024
    s, q = quant(dt)(synth(330 + dt, N * K, 0.02).reshape(N, K))
    qd, sd = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    A = torch.from_numpy(synth(331 + dt, 4 * K, 1.0).reshape(4, K)).cuda()
    A[2, ::5] *= 800.0                    # the exact fix-up pass runs too
    C = torch.empty(4, N, device="cuda")
    noalloc(gpu, A, qd, sd, C, dt)        # set-up call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        noalloc(gpu, A, qd, sd, C, dt)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    ref = torch.empty(4, N, device="cuda")
    gpu.matmul_q_dev(A, qd, sd, ref, dt)
    torch.cuda.synchronize()
    assert np.array_equal(C.cpu().numpy(), ref.cpu().numpy())


def test_noalloc_k0_gives_zeros_like_the_regular_entry(gpu):
    """K = 0: no products, C = 0 whatever the scales hold (the regular entry
    point zero-fills without reading B_s)."""
    q = torch.zeros(4, 16, dtype=torch.int8, device="cuda")
    sc = torch.full((4,), float("nan"), device="cuda")
    A = torch.zeros(3, 16, device="cuda")
    got = torch.full((3, 4), 7.0, device="cuda")
    ref = torch.full((3, 4), 7.0, device="cuda")
    gpu.check(gpu.lib().moe_matmul_q_dev_noalloc(A.data_ptr(), q.data_ptr(), sc.data_ptr(), got.data_ptr(),
                                                 3, 4, 0, 2, None))
    gpu.check(gpu.lib().moe_matmul_q8_dev(A.data_ptr(), q.data_ptr(), sc.data_ptr(), ref.data_ptr(), 3, 4, 0, None))
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), ref.cpu().numpy())
    assert not got.cpu().numpy().any()


def test_noalloc_rejects_sizes_beyond_its_scratch(gpu):
    """Fast-path shapes beyond the fixed array are refused before any work
    (B_q = NULL is 16-byte aligned, so these shapes take the fast path)."""
    lib = gpu.lib()
    rc = lib.moe_matmul_q_dev_noalloc(None, None, None, None, 4097, 8, 64, 2, None)
    assert rc == gpu.MOE_ERR_INVALID and b"scratch" in lib.moe_cuda_last_error()
    rc = lib.moe_matmul_q_dev_noalloc(None, None, None, None, 300, 8, 2048, 2, None)
    assert rc == gpu.MOE_ERR_INVALID
