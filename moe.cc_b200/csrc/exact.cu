// exact.cu — the expert FFN with int32 activations of any magnitude, for
// the calls the fast kernels refuse (an activation outside their integer
// range, or NaN/inf: kErrRange). One thread per output, the reference's
// arithmetic step for step (test_model_trace.c:489-503 with kernels.c:51-128):
//   g = matmul(x, W_g[e]), u = matmul(x, W_u[e]), h = silu(g) * u,
//   y = matmul(h, W_d[e]), matmul = ((float)Σ trunc(a*S)·q / S) * s[row].
// Slots are s = t*K + k (the routing of the refused call); y is written in
// that layout for the k-ordered combine.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.cuh"

namespace moe {
namespace {

// Σ_k trunc(a[k]*S) * w[k] over one weight row, in int32 (two's-complement
// wrap, as the reference's int32 accumulator).
template <int DT>
__device__ __forceinline__ int exact_row_dot(const float* __restrict__ a, const uint8_t* __restrict__ w, int K) {
  unsigned acc = 0;
  if (DT == 8) {
    const int8_t* ws = reinterpret_cast<const int8_t*>(w);
    for (int k = 0; k < K; ++k) acc += (unsigned)(trunc_scale(__ldg(a + k), 127.0f) * (int)__ldg(ws + k));
  } else {
    for (int k = 0; k < K; k += 2) {
      const uint8_t b = __ldg(w + (k >> 1));
      acc += (unsigned)(trunc_scale(__ldg(a + k), 7.0f) * ((int)(b & 0xF) - 8));
      acc += (unsigned)(trunc_scale(__ldg(a + k + 1), 7.0f) * ((int)(b >> 4) - 8));
    }
  }
  return (int)acc;
}

struct ExactArgs {
  const uint8_t* slab;
  size_t stride, gq_off, uq_off, dq_off, gs_off, us_off, ds_off;
  int D, F, K, TK, e_begin, E_local, gu_rb, d_rb;
  const float* xn;   // [T][D]
  const int* idx;    // [T*K]
  float* h;          // [T*K][F]
  float* y;          // [T*K][D]
};

// one thread per (slot, expert row f): h[s][f] = silu(g_f) * u_f
template <int DT>
__global__ void exact_gateup_kernel(const ExactArgs a) {
  const long c = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= (long)a.TK * a.F) return;
  const int s = (int)(c / a.F), f = (int)(c % a.F), t = s / a.K;
  const int e = a.idx[s] - a.e_begin;
  if (e < 0 || e >= a.E_local) { a.h[c] = __int_as_float(0x7fffffff); return; }   // no expert (NaN logits)
  const uint8_t* base = a.slab + (size_t)e * a.stride;
  const float* x = a.xn + (size_t)t * a.D;
  const float g = fmul(div_qscale(exact_row_dot<DT>(x, base + a.gq_off + (size_t)f * a.gu_rb, a.D), DT == 8),
                       reinterpret_cast<const float*>(base + a.gs_off)[f]);
  const float u = fmul(div_qscale(exact_row_dot<DT>(x, base + a.uq_off + (size_t)f * a.gu_rb, a.D), DT == 8),
                       reinterpret_cast<const float*>(base + a.us_off)[f]);
  a.h[c] = fmul(silu_ref(g), u);
}

// one thread per (slot, output row d): y[s][d] = (W_d[e] h_s)[d]
template <int DT>
__global__ void exact_down_kernel(const ExactArgs a) {
  const long c = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= (long)a.TK * a.D) return;
  const int s = (int)(c / a.D), d = (int)(c % a.D);
  const int e = a.idx[s] - a.e_begin;
  if (e < 0 || e >= a.E_local) { a.y[c] = __int_as_float(0x7fffffff); return; }
  const uint8_t* base = a.slab + (size_t)e * a.stride;
  a.y[c] = fmul(div_qscale(exact_row_dot<DT>(a.h + (size_t)s * a.F, base + a.dq_off + (size_t)d * a.d_rb, a.F),
                           DT == 8),
                reinterpret_cast<const float*>(base + a.ds_off)[d]);
}

}  // namespace

void launch_exact_experts(const LayerDev& L, const float* xn, const int* idx, int T, float* h, float* y,
                          cudaStream_t st) {
  ExactArgs a{};
  a.slab = L.slab; a.stride = L.expert_stride;
  a.gq_off = L.gq_off; a.uq_off = L.uq_off; a.dq_off = L.dq_off;
  a.gs_off = L.gs_off; a.us_off = L.us_off; a.ds_off = L.ds_off;
  a.D = L.D; a.F = L.F; a.K = L.topk; a.TK = T * L.topk; a.e_begin = L.e_begin; a.E_local = L.e_end - L.e_begin;
  a.gu_rb = L.gu_rb; a.d_rb = L.d_rb;
  a.xn = xn; a.idx = idx; a.h = h; a.y = y;
  const long n1 = (long)a.TK * a.F, n2 = (long)a.TK * a.D;
  if (n1 <= 0) return;
  if (L.dtype == 2) {
    exact_gateup_kernel<8><<<(unsigned)((n1 + 127) / 128), 128, 0, st>>>(a);
    exact_down_kernel<8><<<(unsigned)((n2 + 127) / 128), 128, 0, st>>>(a);
  } else {
    exact_gateup_kernel<4><<<(unsigned)((n1 + 127) / 128), 128, 0, st>>>(a);
    exact_down_kernel<4><<<(unsigned)((n2 + 127) / 128), 128, 0, st>>>(a);
  }
}

}  // namespace moe
