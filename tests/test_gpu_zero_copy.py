"""Host-pointer moe_ffn on page-locked buffers (the zero-copy path of
runtime.cu: the combine reads and updates x_inout through its mapped address
and writes the top-k lists and the error word straight to host memory) must
return exactly what the same call returns on pageable buffers (the copy
path): outputs, top-k indices and weights bit for bit, on every expert path
(GEMV T=1, fused T=16, prefill T=512, fp32 experts), with out-of-range
activations (exact fix-up), an unaligned x_inout (scalar combine), a given
routing, and pageable top-k outputs beside a pinned x_inout (copy path)."""
import numpy as np
import pytest

from helpers import synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

_L = {}


def layer(gpu, dt):
    if dt not in _L:
        import synth as sy
        Ld = sy.make_layer_dev(torch, 7, 0, 128, 2048, 768, dt, bias=dt == 3)
        torch.cuda.synchronize()
        gpu.upload_layer(700 + dt, Ld, device_arrays=True)
        gpu.check_status()
        _L[dt] = 700 + dt
    return _L[dt]


def pinned(a):
    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


def call_pinned(gpu, lid, xn, xo, K=8, pin_topk=True, given=None, offset=0):
    """moe_ffn with host pointers into page-locked tensors; offset: floats
    by which x_inout starts into its pinned buffer (misaligns it)."""
    T, D = xn.shape
    xn_t = pinned(xn)
    buf = torch.zeros(T * D + offset + 4, dtype=torch.float32).pin_memory()
    buf[offset:offset + T * D] = torch.from_numpy(xo.ravel())
    flags = gpu.HOST_PTRS
    if given is not None:
        idx, p = given[0].astype(np.int32).copy(), given[1].astype(np.float32).copy()
        flags |= gpu.GIVEN_TOPK
    else:
        idx, p = np.empty((T, K), np.int32), np.empty((T, K), np.float32)
    if pin_topk:
        idx_t, p_t = pinned(idx), pinned(p)
        ip, pp = idx_t.data_ptr(), p_t.data_ptr()
    else:
        ip, pp = idx.ctypes.data, p.ctypes.data
    gpu.check(gpu.lib().moe_ffn(lid, xn_t.data_ptr(), buf.data_ptr() + 4 * offset, T, ip, pp, flags, None))
    gpu.check_status()
    out = buf[offset:offset + T * D].numpy().reshape(T, D).copy()
    if pin_topk:
        idx, p = idx_t.numpy(), p_t.numpy()
    return out, idx, p


def same(a, b):
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("dt,T", [(2, 1), (2, 16), (3, 16), (3, 512), (2, 512)])
def test_pinned_equals_pageable(gpu, dt, T):
    lid = layer(gpu, dt)
    xn = synth(9100 + T + dt, T * 2048, 1.0).reshape(T, 2048)
    xo = synth(9200 + T + dt, T * 2048, 1.0).reshape(T, 2048)
    want = gpu.moe_ffn_host(lid, xn, xo)
    got = call_pinned(gpu, lid, xn, xo)
    for w, g_, name in zip(want, got, ("x", "idx", "p")):
        assert same(np.asarray(w), np.asarray(g_)), name


def test_pinned_out_of_range_unaligned_and_fallbacks(gpu):
    lid = layer(gpu, 2)
    T = 16
    xn = synth(9300, T * 2048, 1.0).reshape(T, 2048)
    xn[::3, ::97] *= 400.0          # beyond the Q8 limbs: exact fix-up
    xo = synth(9301, T * 2048, 1.0).reshape(T, 2048)
    want = gpu.moe_ffn_host(lid, xn, xo)
    for kw in ({}, {"offset": 1}, {"pin_topk": False}):
        got = call_pinned(gpu, lid, xn, xo, **kw)
        for w, g_, name in zip(want, got, ("x", "idx", "p")):
            assert same(np.asarray(w), np.asarray(g_)), (kw, name)
    # a given routing: no top-k outputs, x_inout still zero-copy
    giv = (want[1], want[2])
    w2 = gpu.moe_ffn_host(lid, xn, xo, given=giv)
    g2 = call_pinned(gpu, lid, xn, xo, given=giv)
    assert same(w2[0], g2[0])


def test_pinned_fp32_experts(gpu):
    E, D, F, T = 16, 256, 128, 5
    n = lambda s, shape, std: synth(s, int(np.prod(shape)), std).reshape(shape)
    gpu.upload_layer_f32(790, n(9400, (E, D), 0.5), None, n(9401, (E, F, D), 0.3), n(9402, (E, F, D), 0.3),
                         n(9403, (E, D, F), 0.3), top_k=4)
    xn = n(9404, (T, D), 1.0)
    xo = n(9405, (T, D), 1.0)
    want = gpu.moe_ffn_host(790, xn, xo, topk=4)
    got = call_pinned(gpu, 790, xn, xo, K=4)
    for w, g_, name in zip(want, got, ("x", "idx", "p")):
        assert same(np.asarray(w), np.asarray(g_)), name
    gpu.free_layer(790)
