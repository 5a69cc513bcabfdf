// f32_experts.cu — the unquantised (fp32) expert FFN, for layers whose
// experts are plain fp32 matrices: model.c's layer_forward_f32
// (model.c:172-187) and the fp32 branch of test_model_trace.c:506-511:
//   g = x · W_g[e]^T; g = silu(g); u = x · W_u[e]^T; g *= u; y = g · W_d[e]^T
// Every output is one sequential fp32 chain in k order (matmul_f32,
// test_model_trace.c:213-227), with IEEE single rounding after each multiply
// and each add and no FMA contraction, so results equal the reference's
// bit for bit; only the order of independent outputs changes.
//
// A CTA owns one slot (token, k) and 128 output rows; 128 threads, one chain
// each. K advances in tiles of 32: the CTA stages the activation tile and the
// 128 x 32 weight tile(s) through shared memory with coalesced loads (each
// warp reads whole 128-byte row segments), then every thread adds its row's
// 32 products in order. The weight tile is padded to 33 floats per row, so
// the threads' column reads hit distinct banks.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.cuh"

namespace moe {
namespace {

constexpr int kRows = 128, kKT = 32, kPad = kKT + 1;

struct F32Args {
  const uint8_t* slab;
  size_t stride, gq_off, uq_off, dq_off;   // fp32 gate [F][D], up [F][D], down [D][F]
  int D, F, K, TK, e_begin, E_local;
  const float* xn;    // [T][D]
  const int* idx;     // [T*K]
  float* h;           // [T*K][F]
  float* y;           // [T*K][D]
};

// GATEUP: rows f of gate and up against x[t]; h = silu(g) * u.
// DOWN:   rows d of down against h[s]; y.
template <bool GATEUP>
__global__ void __launch_bounds__(kRows) f32_expert_kernel(const F32Args a) {
  __shared__ float xs[kKT];
  __shared__ float w0[kRows][kPad];
  __shared__ float w1[GATEUP ? kRows : 1][kPad];
  pdl_wait();
  pdl_launch();
  const int s = blockIdx.y, t = s / a.K;
  const int N = GATEUP ? a.F : a.D, Kd = GATEUP ? a.D : a.F;
  const int r0 = blockIdx.x * kRows, tid = threadIdx.x;
  const int e = a.idx[s] - a.e_begin;
  float* out = GATEUP ? a.h + (size_t)s * a.F : a.y + (size_t)s * a.D;
  if (e < 0 || e >= a.E_local) {          // no expert for this slot (all logits NaN/-inf)
    if (r0 + tid < N) out[r0 + tid] = 0.0f;
    return;
  }
  const uint8_t* ex = a.slab + (size_t)e * a.stride;
  const float* W0 = reinterpret_cast<const float*>(ex + (GATEUP ? a.gq_off : a.dq_off));
  const float* W1 = reinterpret_cast<const float*>(ex + a.uq_off);
  const float* x = GATEUP ? a.xn + (size_t)t * a.D : a.h + (size_t)s * a.F;
  float acc0 = 0.0f, acc1 = 0.0f;
  for (int k0 = 0; k0 < Kd; k0 += kKT) {
    const int kn = min(kKT, Kd - k0);
    if (tid < kKT) xs[tid] = tid < kn ? x[k0 + tid] : 0.0f;
    for (int i = tid; i < kRows * kKT; i += kRows) {
      const int rr = i / kKT, c = i % kKT, row = r0 + rr;
      const bool in = row < N && c < kn;
      w0[rr][c] = in ? __ldg(W0 + (size_t)row * Kd + k0 + c) : 0.0f;
      if (GATEUP) w1[rr][c] = in ? __ldg(W1 + (size_t)row * Kd + k0 + c) : 0.0f;
    }
    __syncthreads();
    for (int c = 0; c < kn; ++c) {
      acc0 = fadd(acc0, fmul(xs[c], w0[tid][c]));
      if (GATEUP) acc1 = fadd(acc1, fmul(xs[c], w1[tid][c]));
    }
    __syncthreads();
  }
  if (r0 + tid >= N) return;
  out[r0 + tid] = GATEUP ? fmul(silu_ref(acc0), acc1) : acc0;
}

}  // namespace

void launch_f32_experts(const LayerDev& L, const float* xn, const int* idx, int T, float* h, float* y,
                        cudaStream_t st) {
  const int TK = T * L.topk;
  if (TK <= 0) return;
  F32Args a{};
  a.slab = L.slab; a.stride = L.expert_stride;
  a.gq_off = L.gq_off; a.uq_off = L.uq_off; a.dq_off = L.dq_off;
  a.D = L.D; a.F = L.F; a.K = L.topk; a.TK = TK; a.e_begin = L.e_begin; a.E_local = L.e_end - L.e_begin;
  a.xn = xn; a.idx = idx; a.h = h; a.y = y;
  launch_pdl(f32_expert_kernel<true>, dim3((L.F + kRows - 1) / kRows, TK), dim3(kRows), 0, st, a);
  launch_pdl(f32_expert_kernel<false>, dim3((L.D + kRows - 1) / kRows, TK), dim3(kRows), 0, st, a);
}

}  // namespace moe
