// exact.cu — the exact fix-up pass of moe_ffn.
//
// The fast expert kernels carry activations as 16-bit (Q8: two byte limbs)
// or 8-bit (Q4) integers. The reference truncates with no range limit,
// (int32_t)(a * 127f) (kernels.c:66) and (int32_t)(a * 7f) (kernels.c:113),
// and accumulates in int32. When a token's activation x, or the activation h
// of one of its slots, falls outside the fast range (or is NaN/inf), the fast
// kernels mark the token (range_fail in common.cuh) and this pass recomputes
// every slot of the marked tokens with int32 activations of any magnitude,
// the reference's arithmetic step for step (test_model_trace.c:494-503 with
// kernels.c:51-128):
//   g = matmul(x, W_g[e]); g = silu(g); u = matmul(x, W_u[e]); h = g * u;
//   y = matmul(h, W_d[e]);   matmul = ((float)Σ trunc(a*S)·q / S) * s[row]
// It writes y where the combine reads it, so the combine that follows gives
// the reference's result for every token.
//
// Launched after the expert kernels of every moe_ffn call. When no token was
// marked, each CTA reads one word and leaves. Otherwise one CTA per slot
// (grid-strided) truncates x into shared memory once, computes h with one
// warp per gate/up row pair, truncates h into shared memory, then y with one
// warp per down row. The last CTA to finish clears the marks.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.cuh"

namespace moe {
namespace {

struct FixArgs {
  const uint8_t* slab;
  size_t stride, gq_off, uq_off, dq_off, gs_off, us_off, ds_off;
  int D, F, K, T, e_begin, E_local, gu_rb, d_rb;
  const float* xn;        // [T][D] the MoE input
  const int* idx;         // [T*K] top-k experts (global ids)
  const int* slot_pos;    // slot -> y row, or null (row = slot)
  float* y;               // [rows][D]
  int* flags;             // [0] any, [1] arrival counter, [2 + t] token t
  int ep_on; EpView ep;   // expert parallel (see launch_exact_fixup)
};

__device__ __forceinline__ uint8_t* ep_peer(const EpView& ep, int p) {
  return reinterpret_cast<uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(ep.base) + p));
}

// Σ_k aq[k] * w[k] over one weight row, one warp, int32 with two's-complement
// wrap (the reference's int32 accumulator; the sum is order-free). Q8: int8
// weights. Q4: nibble pairs, low nibble = even k, value = nibble - 8
// (kernels.c:110-125). aq is 16-byte aligned shared memory; K is a multiple
// of 4 (Q8) or 8 (Q4), and w is 4-byte aligned.
template <int DT>
__device__ __forceinline__ int warp_row_dot(const int* aq, const uint8_t* __restrict__ w, int K, int lane) {
  unsigned acc = 0;
  if (DT == 8) {
    for (int k = lane * 4; k < K; k += 128) {
      const int wv = __ldg(reinterpret_cast<const int*>(w + k));
      const int4 av = *reinterpret_cast<const int4*>(aq + k);
      acc += (unsigned)(av.x * ((wv << 24) >> 24)) + (unsigned)(av.y * ((wv << 16) >> 24)) +
             (unsigned)(av.z * ((wv << 8) >> 24)) + (unsigned)(av.w * (wv >> 24));
    }
  } else {
    for (int k = lane * 8; k < K; k += 256) {
      const unsigned wv = __ldg(reinterpret_cast<const unsigned*>(w + k / 2));
      const int4 a0 = *reinterpret_cast<const int4*>(aq + k);
      const int4 a1 = *reinterpret_cast<const int4*>(aq + k + 4);
      const int av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) acc += (unsigned)(av[i] * ((int)((wv >> (4 * i)) & 0xFu) - 8));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return (int)acc;
}

constexpr int kFixThreads = 256;

template <int DT>
__global__ void __launch_bounds__(kFixThreads) exact_fixup_kernel(const FixArgs a) {
  extern __shared__ __align__(16) int fsm[];
  int* xq = fsm;                 // [D] truncated x of the slot's token
  int* hq = fsm + a.D;           // [F] truncated h of the slot
  __shared__ int s_any, s_last;
  constexpr float S = DT == 8 ? 127.0f : 7.0f;
  const int seq32 = (int)a.ep.seq;
  pdl_wait();
  pdl_launch();
  // flags[0]: some token was marked, here or (expert parallel: copied by the
  // routing kernel from every rank's xflag) by its home rank. Otherwise the
  // expert kernels have raised the combine flags already.
  if (threadIdx.x == 0) s_any = *reinterpret_cast<volatile int*>(a.flags);
  __syncthreads();
  if (!s_any) return;            // nothing marked: every CTA leaves here

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kFixThreads / 32;
  for (int s = blockIdx.x; s < a.T * a.K; s += gridDim.x) {
    const int t = s / a.K;
    const float* x = a.xn + (size_t)t * a.D;
    float* yr = a.y + (size_t)(a.slot_pos ? a.slot_pos[s] : s) * a.D;
    bool marked = a.flags[2 + t] != 0;
    if (a.ep_on) {
      // token t lives on rank h as its local token tl
      const int h = t / a.ep.T_local, tl = t - h * a.ep.T_local;
      const uint8_t* hb = ep_peer(a.ep, h);
      marked = marked || reinterpret_cast<const int*>(hb + a.ep.xflag_off)[2 + tl] == seq32;
      x = reinterpret_cast<const float*>(hb + a.ep.xf_off) + (size_t)tl * a.D;
      yr = reinterpret_cast<float*>(ep_peer(a.ep, h) + a.ep.y_off) + (size_t)(s - h * a.ep.T_local * a.K) * a.D;
    }
    if (!marked) continue;
    const int e = a.idx[s] - a.e_begin;
    if (e < 0 || e >= a.E_local) continue;     // another rank's expert, or no expert (all logits NaN/-inf)
    const uint8_t* ex = a.slab + (size_t)e * a.stride;
    for (int k = threadIdx.x; k < a.D; k += kFixThreads) xq[k] = trunc_scale(x[k], S);
    __syncthreads();
    const float* gs = reinterpret_cast<const float*>(ex + a.gs_off);
    const float* us = reinterpret_cast<const float*>(ex + a.us_off);
    for (int f = warp; f < a.F; f += nw) {
      const int dg = warp_row_dot<DT>(xq, ex + a.gq_off + (size_t)f * a.gu_rb, a.D, lane);
      const int du = warp_row_dot<DT>(xq, ex + a.uq_off + (size_t)f * a.gu_rb, a.D, lane);
      if (lane == 0) {
        const float g = fmul(div_qscale(dg, DT == 8), __ldg(gs + f));
        const float u = fmul(div_qscale(du, DT == 8), __ldg(us + f));
        hq[f] = trunc_scale(fmul(silu_ref(g), u), S);
      }
    }
    __syncthreads();
    const float* ds = reinterpret_cast<const float*>(ex + a.ds_off);
    for (int d = warp; d < a.D; d += nw) {
      const int dd = warp_row_dot<DT>(hq, ex + a.dq_off + (size_t)d * a.d_rb, a.F, lane);
      if (lane == 0) yr[d] = fmul(div_qscale(dd, DT == 8), __ldg(ds + d));
    }
    __syncthreads();             // xq / hq are rewritten by the next slot
  }

  // The last CTA out clears the local marks for the next call and,
  // expert-parallel, raises this rank's combine flag at every rank (release
  // after a system fence: a rank that sees the flag sees every y row this
  // rank stored, from the expert kernels and from this pass; the expert
  // kernels left the flags to this pass because a token was marked).
  __syncthreads();
  if (threadIdx.x == 0) {
    if (a.ep_on) __threadfence_system(); else __threadfence();
    s_last = atomicAdd(a.flags + 1, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    for (int i = 2 + threadIdx.x; i < 2 + a.T; i += kFixThreads) a.flags[i] = 0;
    __syncthreads();
    if (threadIdx.x == 0) {
      a.flags[0] = 0;
      a.flags[1] = 0;
      if (a.ep_on) ep_raise_combine(a.ep);
    }
  }
}

}  // namespace

void launch_exact_fixup(const LayerDev& L, const float* xn, const int* idx, const int* slot_pos, int T,
                        float* y, int* flags, int sm_count, cudaStream_t st, const EpView* ep) {
  const int TK = T * L.topk;
  if (TK <= 0 || !flags) return;
  FixArgs a{};
  a.slab = L.slab; a.stride = L.expert_stride;
  a.gq_off = L.gq_off; a.uq_off = L.uq_off; a.dq_off = L.dq_off;
  a.gs_off = L.gs_off; a.us_off = L.us_off; a.ds_off = L.ds_off;
  a.D = L.D; a.F = L.F; a.K = L.topk; a.T = T; a.e_begin = L.e_begin; a.E_local = L.e_end - L.e_begin;
  a.gu_rb = L.gu_rb; a.d_rb = L.d_rb;
  a.xn = xn; a.idx = idx; a.slot_pos = slot_pos; a.y = y; a.flags = flags;
  a.ep_on = ep != nullptr;
  if (ep) a.ep = *ep;
  const int grid = TK < 2 * sm_count ? TK : 2 * sm_count;
  const size_t smem = sizeof(int) * ((size_t)L.D + L.F);
  auto go = [&](auto kern) {
    static size_t attr = 48 * 1024;
    if (smem > attr && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
                           cudaSuccess)
      attr = smem;
    launch_pdl(kern, dim3(grid), dim3(kFixThreads), smem, st, a);
  };
  if (L.dtype == 2) go(exact_fixup_kernel<8>);
  else go(exact_fixup_kernel<4>);
}

}  // namespace moe
