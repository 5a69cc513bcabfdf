"""ctypes binding of libmoe_cuda.so (the C-ABI in include/moe_cuda.h).

This is the Python face of the same boundary a C host links against: the
reference-shaped entry points (matmul_f32_q8 / matmul_f32_q4 / matmul_adaptive,
kernels.c:51,96,149) plus the fused moe_ffn block and its residency API.
Host numpy arrays go through the synchronous host-pointer entries; torch CUDA
tensors go through the device-pointer entries (pointers and a stream only —
torch is plumbing for device memory, never part of the computation).

There is no CPU fallback: if the library is missing or no GPU is present the
calls fail loudly.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_cuda.so")

MOE_OK, MOE_ERR_INVALID, MOE_ERR_CUDA, MOE_ERR_NOT_INIT = 0, 1, 2, 3
MOE_ERR_RANGE, MOE_ERR_UNSUPPORTED, MOE_ERR_NOMEM = 4, 5, 6
Q8, Q4 = 2, 3
HOST_PTRS, DEVICE_PTRS, FORCE_GEMV, FORCE_GEMM = 0x1, 0x0, 0x4, 0x8
SEQ_RESIDUAL, GIVEN_TOPK = 0x10, 0x20
F32 = 0

# Every symbol include/moe_cuda.h declares (checked by the CPU test suite).
EXPORTS = (
    "moe_cuda_init", "moe_cuda_shutdown", "moe_cuda_last_error", "moe_cuda_check_status",
    "matmul_f32_q8", "matmul_f32_q4", "matmul_adaptive",
    "moe_matmul_q8_dev", "moe_matmul_q4_dev", "moe_matmul_f32_dev", "moe_matmul_batched_dev",
    "moe_quantize_rowwise_q8_dev", "moe_quantize_rowwise_q4_dev",
    "moe_cuda_upload_layer", "moe_cuda_upload_layer_dev", "moe_cuda_upload_layer_f32", "moe_cuda_free_layer",
    "moe_cuda_layer_bytes", "moe_ffn", "moe_ffn_partial", "moe_ffn_combine",
    "moe_synth_normal_host", "moe_synth_normal_dev",
    "moe_cuda_profile", "moe_cuda_profile_read", "moe_matmul_q_dev_noalloc",
    "moe_cuda_ep_setup", "moe_cuda_ep_connect", "moe_ffn_ep",
    "moe_bin_layer_info", "moe_cuda_load_bin_layer",
    "moe_bin_open", "moe_bin_close", "moe_bin_find", "moe_bin_read",
    "moe_bin_layer_info_h", "moe_cuda_load_bin_layer_h",
    "moe_bin_create", "moe_bin_put", "moe_bin_finish",
    "moe_quantize_rowwise_q8_host", "moe_quantize_rowwise_q4_host",
)


class MoeError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"libmoe_cuda error {code}: {msg}")
        self.code = code


class QuantizedWeight(C.Structure):
    """model.h:26-32."""
    _fields_ = [("q", C.c_void_p), ("s", C.c_void_p), ("rows", C.c_int),
                ("cols", C.c_int), ("dtype", C.c_int)]


_lib = None


def lib():
    """Load libmoe_cuda.so (built in-tree by `make -C moe.cc_b200`)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MoeError(MOE_ERR_NOT_INIT, f"{LIB_PATH} is not built (run make -C moe.cc_b200)")
        L = C.CDLL(LIB_PATH)
        vp, i, sz, u64, f = C.c_void_p, C.c_int, C.c_size_t, C.c_uint64, C.c_float
        sig = {
            "moe_cuda_init": ([i, i, i, vp], i), "moe_cuda_shutdown": ([], i),
            "moe_cuda_last_error": ([], C.c_char_p), "moe_cuda_check_status": ([], i),
            "matmul_f32_q8": ([vp, vp, vp, vp, i, i, i], None),
            "matmul_f32_q4": ([vp, vp, vp, vp, i, i, i], None),
            "matmul_adaptive": ([vp, vp, vp, vp, i, i, i], None),
            "moe_matmul_q8_dev": ([vp, vp, vp, vp, i, i, i, vp], i),
            "moe_matmul_q4_dev": ([vp, vp, vp, vp, i, i, i, vp], i),
            "moe_matmul_f32_dev": ([vp, vp, vp, i, i, i, vp], i),
            "moe_matmul_batched_dev": ([vp, vp, vp, vp, i, i, i, i, vp], i),
            "moe_quantize_rowwise_q8_dev": ([vp, i, i, vp, vp, vp], i),
            "moe_quantize_rowwise_q4_dev": ([vp, i, i, vp, vp, vp], i),
            "moe_cuda_upload_layer": ([i, vp, vp, vp, vp, vp, i], i),
            "moe_cuda_upload_layer_dev": ([i, vp, vp, vp, vp, vp, i], i),
            "moe_cuda_upload_layer_f32": ([i, vp, vp, vp, vp, vp, i, i, i, i], i),
            "moe_cuda_free_layer": ([i], i), "moe_cuda_layer_bytes": ([i], sz),
            "moe_ffn": ([i, vp, vp, i, vp, vp, i, vp], i),
            "moe_ffn_partial": ([i, vp, i, vp, vp, vp, vp], i),
            "moe_ffn_combine": ([vp, vp, vp, i, i, i, vp], i),
            "moe_synth_normal_host": ([u64, u64, sz, f, vp], None),
            "moe_synth_normal_dev": ([u64, u64, sz, f, vp, vp], i),
            "moe_cuda_profile": ([i], i),
            "moe_matmul_q_dev_noalloc": ([vp, vp, vp, vp, i, i, i, i, vp], i),
            "moe_cuda_profile_read": ([i, vp, i, vp, vp], i),
            "moe_cuda_ep_setup": ([i, i, i, vp], i),
            "moe_cuda_ep_connect": ([vp], i),
            "moe_ffn_ep": ([i, vp, i, vp, vp], i),
            "moe_bin_layer_info": ([C.c_char_p, i, vp, vp, vp, vp, vp], i),
            "moe_cuda_load_bin_layer": ([C.c_char_p, i, i], i),
            "moe_bin_open": ([C.c_char_p], vp), "moe_bin_close": ([vp], None),
            "moe_bin_find": ([vp, C.c_char_p, vp, vp, vp, vp], i),
            "moe_bin_read": ([vp, C.c_char_p, vp, sz], i),
            "moe_bin_layer_info_h": ([vp, i, vp, vp, vp, vp, vp], i),
            "moe_cuda_load_bin_layer_h": ([vp, i, i], i),
            "moe_bin_create": ([C.c_char_p, C.c_uint32], vp), "moe_bin_put": ([vp, C.c_char_p, i, i, vp, vp], i),
            "moe_bin_finish": ([vp], i),
            "moe_quantize_rowwise_q8_host": ([vp, i, i, vp, vp], i),
            "moe_quantize_rowwise_q4_host": ([vp, i, i, vp, vp], i),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes, fn.restype = args, res
        _lib = L
    return _lib


def check(rc):
    if rc != MOE_OK:
        raise MoeError(rc, lib().moe_cuda_last_error().decode(errors="replace"))
    return rc


def _p(a):
    """Raw pointer of a numpy array or torch tensor (None passes through)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags.c_contiguous
        return a.ctypes.data
    assert a.is_contiguous()
    return a.data_ptr()


def _stream(s):
    if s is None:
        return None
    return getattr(s, "cuda_stream", s)


def init(device=0, ep_world=1, ep_rank=0):
    check(lib().moe_cuda_init(device, ep_world, ep_rank, None))


def shutdown():
    check(lib().moe_cuda_shutdown())


def check_status():
    check(lib().moe_cuda_check_status())


# ---- reference-shaped host API (kernels.c) --------------------------------

def matmul_f32_q8(A, Bq, Bs, N, K):
    A = np.ascontiguousarray(A, np.float32).reshape(-1, K)
    out = np.empty((A.shape[0], N), np.float32)
    lib().matmul_f32_q8(_p(A), _p(Bq), _p(Bs), _p(out), A.shape[0], N, K)
    return out


def matmul_f32_q4(A, Bq, Bs, N, K):
    A = np.ascontiguousarray(A, np.float32).reshape(-1, K)
    out = np.empty((A.shape[0], N), np.float32)
    lib().matmul_f32_q4(_p(A), _p(Bq), _p(Bs), _p(out), A.shape[0], N, K)
    return out


def matmul_adaptive(A, W_fp32, W_q, N, K):
    """W_q: None (fp32 path) or a QuantizedWeight."""
    A = np.ascontiguousarray(A, np.float32).reshape(-1, K)
    out = np.empty((A.shape[0], N), np.float32)
    lib().matmul_adaptive(_p(A), _p(W_fp32), None if W_q is None else C.addressof(W_q),
                          _p(out), A.shape[0], N, K)
    return out


# ---- device API ------------------------------------------------------------

def matmul_q_dev(A, Bq, Bs, C_out, dtype, stream=None):
    M, K = A.shape
    N = C_out.shape[1]
    fn = lib().moe_matmul_q8_dev if dtype == Q8 else lib().moe_matmul_q4_dev
    check(fn(_p(A), _p(Bq), _p(Bs), _p(C_out), M, N, K, _stream(stream)))


def quantize_rowwise_dev(W, q, s, dtype, stream=None):
    rows, cols = W.shape
    fn = lib().moe_quantize_rowwise_q8_dev if dtype == Q8 else lib().moe_quantize_rowwise_q4_dev
    check(fn(_p(W), rows, cols, _p(q), _p(s), _stream(stream)))


def synth_normal_host(seed, n, std=1.0, offset=0):
    out = np.empty(n, np.float32)
    lib().moe_synth_normal_host(seed, offset, n, std, _p(out))
    return out


def synth_normal_dev(seed, out, std=1.0, offset=0, stream=None):
    check(lib().moe_synth_normal_dev(seed, offset, out.numel(), std, _p(out), _stream(stream)))


def _qw_array(q, s, rows, cols, dtype):
    """QuantizedWeight[E] over contiguous per-expert arrays q [E][rows][*], s [E][rows]."""
    E = q.shape[0]
    arr = (QuantizedWeight * E)()
    qb, sb = _p(q), _p(s)
    qstride = q[0].nbytes if isinstance(q, np.ndarray) else q[0].numel() * q.element_size()
    for e in range(E):
        arr[e].q = qb + e * qstride
        arr[e].s = sb + e * rows * 4
        arr[e].rows, arr[e].cols, arr[e].dtype = rows, cols, dtype
    return arr


def upload_layer(layer, L, device_arrays=False):
    """L: dict with dtype, router_w [E][D], router_b or None, gq/uq [E][F][*],
    gs/us [E][F], dq [E][D][*], ds [E][D] (numpy, or torch CUDA tensors with
    device_arrays=True). Keeps the QuantizedWeight arrays alive on L."""
    E, D = L["router_w"].shape
    F = L["gs"].shape[1]
    dt = L["dtype"]
    g = _qw_array(L["gq"], L["gs"], F, D, dt)
    u = _qw_array(L["uq"], L["us"], F, D, dt)
    d = _qw_array(L["dq"], L["ds"], D, F, dt)
    L["_qw"] = (g, u, d)
    fn = lib().moe_cuda_upload_layer_dev if device_arrays else lib().moe_cuda_upload_layer
    check(fn(layer, C.addressof(g), C.addressof(u), C.addressof(d), _p(L["router_w"]),
             _p(L.get("router_b")), E))


def bin_layer_info(path, src_layer):
    """(E, D, F, dtype, has_bias) of one layer of a .bin weight file."""
    v = [C.c_int(0) for _ in range(5)]
    check(lib().moe_bin_layer_info(os.fsencode(path), src_layer, *[C.byref(x) for x in v]))
    return tuple(x.value for x in v)


class BinFile:
    """An open .bin weight file (moe_bin_open): find(name) -> (dtype, shape,
    nbytes), read(name) -> numpy array."""
    _NP = {0: np.float32, 1: np.float16, 2: np.int8, 3: np.uint8}

    def __init__(self, path):
        self.h = lib().moe_bin_open(os.fsencode(path))
        if not self.h:
            raise MoeError(MOE_ERR_INVALID, lib().moe_cuda_last_error().decode(errors="replace"))

    def close(self):
        if self.h:
            lib().moe_bin_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def find(self, name):
        dt, nd, nb = C.c_int(0), C.c_int(0), C.c_size_t(0)
        shape = (C.c_int * 8)()
        check(lib().moe_bin_find(self.h, name.encode(), C.byref(dt), C.byref(nd), shape, C.byref(nb)))
        return dt.value, tuple(shape[:nd.value]), nb.value

    def read(self, name):
        dt, shape, nb = self.find(name)
        out = np.empty(shape, self._NP[dt])
        check(lib().moe_bin_read(self.h, name.encode(), out.ctypes.data, nb))
        return out

    def layer_info(self, src_layer):
        v = [C.c_int(0) for _ in range(5)]
        check(lib().moe_bin_layer_info_h(self.h, src_layer, *[C.byref(x) for x in v]))
        return tuple(x.value for x in v)

    def load_layer(self, src_layer, layer):
        check(lib().moe_cuda_load_bin_layer_h(self.h, src_layer, layer))


def quantize_rowwise_host(W, dtype):
    """(s, q) of export._rowwise_q8 / _q4 on the host (moe_quantize_rowwise_*_host)."""
    W = np.ascontiguousarray(W, np.float32)
    rows, cols = W.shape
    s = np.empty(rows, np.float32)
    if dtype == Q8:
        q = np.empty((rows, cols), np.int8)
        check(lib().moe_quantize_rowwise_q8_host(W.ctypes.data, rows, cols, q.ctypes.data, s.ctypes.data))
    else:
        q = np.empty((rows, cols // 2), np.uint8)
        check(lib().moe_quantize_rowwise_q4_host(W.ctypes.data, rows, cols, q.ctypes.data, s.ctypes.data))
    return s, q


class BinWriter:
    """moe_bin_create / moe_bin_put / moe_bin_finish."""
    _DT = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.int8): 2, np.dtype(np.uint8): 3}

    def __init__(self, path, count):
        self.h = lib().moe_bin_create(os.fsencode(path), count)
        if not self.h:
            raise MoeError(MOE_ERR_INVALID, lib().moe_cuda_last_error().decode(errors="replace"))

    def put(self, name, a):
        a = np.require(a, requirements="C")   # keeps 0-d arrays 0-d
        shape = (C.c_int * max(1, a.ndim))(*a.shape)
        check(lib().moe_bin_put(self.h, name.encode(), self._DT[a.dtype], a.ndim, shape, a.ctypes.data))

    def finish(self):
        h, self.h = self.h, None
        check(lib().moe_bin_finish(h))


def load_bin_layer(path, src_layer, layer):
    """Makes layer `src_layer` of a .bin weight file resident as `layer`."""
    check(lib().moe_cuda_load_bin_layer(os.fsencode(path), src_layer, layer))


def free_layer(layer):
    check(lib().moe_cuda_free_layer(layer))


def layer_bytes(layer):
    return lib().moe_cuda_layer_bytes(layer)


def moe_ffn_host(layer, x_norm2, x_after, topk=8, flags=0, given=None):
    """Host-pointer moe_ffn: returns (x_out, topk_idx, topk_p). given: an
    (idx, p) routing to use (MOE_FFN_GIVEN_TOPK)."""
    x_norm2 = np.ascontiguousarray(x_norm2, np.float32)
    x = np.array(x_after, np.float32, copy=True, order="C")
    T = x.shape[0]
    if given is not None:
        idx = np.ascontiguousarray(given[0], np.int32)
        p = np.ascontiguousarray(given[1], np.float32)
        flags |= GIVEN_TOPK
    else:
        idx = np.empty((T, topk), np.int32)
        p = np.empty((T, topk), np.float32)
    check(lib().moe_ffn(layer, _p(x_norm2), _p(x), T, _p(idx), _p(p), HOST_PTRS | flags, None))
    return x, idx, p


def upload_layer_f32(layer, router_w, router_b, gate, up, down, top_k=8):
    """fp32 experts: gate/up [E][F][D], down [E][D][F] host arrays
    (moe_cuda_upload_layer_f32)."""
    gate, up, down = (np.ascontiguousarray(a, np.float32) for a in (gate, up, down))
    E, F, D = gate.shape
    arr = C.c_void_p * E
    ptrs = [arr(*[a[e].ctypes.data for e in range(E)]) for a in (gate, up, down)]
    router_w = np.ascontiguousarray(router_w, np.float32)
    router_b = None if router_b is None else np.ascontiguousarray(router_b, np.float32)
    check(lib().moe_cuda_upload_layer_f32(layer, ptrs[0], ptrs[1], ptrs[2], _p(router_w), _p(router_b),
                                          E, D, F, top_k))


def moe_ffn_dev(layer, x_norm2, x_inout, topk_idx=None, topk_p=None, flags=0, stream=None):
    """Device-pointer moe_ffn (torch CUDA tensors), asynchronous on `stream`."""
    check(lib().moe_ffn(layer, _p(x_norm2), _p(x_inout), x_norm2.shape[0], _p(topk_idx),
                        _p(topk_p), flags & ~HOST_PTRS, _stream(stream)))


def moe_ffn_partial(layer, x_norm2, y_slots, topk_idx=None, topk_p=None, stream=None):
    check(lib().moe_ffn_partial(layer, _p(x_norm2), x_norm2.shape[0], _p(y_slots),
                                _p(topk_idx), _p(topk_p), _stream(stream)))


def moe_ffn_combine(y_slots, topk_p, x_inout, topk=8, stream=None):
    T, D = x_inout.shape
    check(lib().moe_ffn_combine(_p(y_slots), _p(topk_p), _p(x_inout), T, D, topk, _stream(stream)))


def ep_setup(max_tokens_local, D, topk=8):
    """Allocate this rank's receive buffer; returns its 64-byte IPC handle."""
    h = C.create_string_buffer(64)
    check(lib().moe_cuda_ep_setup(max_tokens_local, D, topk, h))
    return h.raw


def ep_connect(handles):
    """handles: every rank's ep_setup() bytes, in rank order."""
    buf = b"".join(handles)
    check(lib().moe_cuda_ep_connect(C.c_char_p(buf)))


def moe_ffn_ep(layer, x_norm2, x_inout, stream=None):
    """Expert-parallel MoE block over this rank's tokens, exchanges fused into
    the kernels (include/moe_cuda.h: moe_ffn_ep)."""
    check(lib().moe_ffn_ep(layer, _p(x_norm2), x_inout.shape[0], _p(x_inout), _stream(stream)))


def profile(enable):
    check(lib().moe_cuda_profile(1 if enable else 0))


def profile_read(max_kernels=32):
    """{kernel name: (total_ms, launches)} accumulated since profile(True)."""
    nl = 64
    names = C.create_string_buffer(max_kernels * nl)
    ms = (C.c_double * max_kernels)()
    cnt = (C.c_long * max_kernels)()
    n = lib().moe_cuda_profile_read(max_kernels, names, nl, ms, cnt)
    raw = names.raw
    return {raw[i * nl:(i + 1) * nl].split(b"\0")[0].decode(): (ms[i], cnt[i]) for i in range(n)}
