// kernels.cu — CUDA-core kernels of libmoe_cuda (sm_100a): activation
// truncation, router, top-k, routing lists, the decode-regime fused expert
// GEMVs (gate/up + SiLU·up, down + k-ordered combine), the plain Q8/Q4 GEMV of
// the matmul_* entry points, rowwise quantisers and the synthetic generator.
//
// Arithmetic follows the reference exactly (kernels.c:51-128,
// test_model_trace.c:213-288, 463-517): activations are truncated to integers
// once per row, dots are exact integer sums (order-free), and every float step
// is one IEEE round-to-nearest op in the reference's order.
#include "common.cuh"
#include "kernels.cuh"

namespace moe {

// --------------------------------------------------------------------------
// geometry of the warp GEMV: a row of `rb` bytes is read by a group of LPR
// lanes, each lane loading `cpl` 16-byte chunks per pass, `np` passes.
// --------------------------------------------------------------------------
struct Geo { int lpr = 0, cpl = 0, np = 0; };

static bool pick_geo(int rb, Geo& g) {
  if (rb <= 0 || rb % 16) return false;
  const int nc = rb / 16;
  if (nc >= 128) {
    if (nc % 32) return false;
    const int per = nc / 32;
    for (int c = 4; c >= 1; --c)
      if (per % c == 0) { g.lpr = 32; g.cpl = c; g.np = per / c; return true; }
    return false;
  }
  for (int l = 1; l <= 32; l <<= 1)
    if (nc % l == 0 && nc / l <= 4) { g.lpr = l; g.cpl = nc / l; g.np = 1; return true; }
  return false;
}

bool fast_geometry_ok(int dtype, int K) {
  Geo g;
  const int rb = dtype == 2 ? K : K / 2;
  if (dtype == 3 && (K & 1)) return false;
  return pick_geo(rb, g);
}

// one 16-byte weight chunk `c` against the activation row `act` (row of K
// logical elements; Q8: lo plane [0,K), hi plane [K,2K); Q4: K permuted bytes)
template <int DT>
__device__ __forceinline__ void chunk_dot(const uint4 w, const uint8_t* act, int K, int c,
                                          int& a0, int& a1) {
  if (DT == 8) {
    const uint4 lo = __ldg(reinterpret_cast<const uint4*>(act + (size_t)c * 16));
    const uint4 hi = __ldg(reinterpret_cast<const uint4*>(act + K + (size_t)c * 16));
    dot16_q8(w, lo, hi, a0, a1);
  } else {
    const uint4 p0 = __ldg(reinterpret_cast<const uint4*>(act + (size_t)c * 32));
    const uint4 p1 = __ldg(reinterpret_cast<const uint4*>(act + (size_t)c * 32 + 16));
    a0 = dot16_q4(w, p0, p1, a0);
  }
}

// combine limb accumulators into the per-lane partial (mod 2^32)
template <int DT>
__device__ __forceinline__ int lane_partial(int a0, int a1) {
  return DT == 8 ? (int)((unsigned)a0 + ((unsigned)a1 << 8)) : a0;
}

template <int LPR>
__device__ __forceinline__ int group_sum(int v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ((float)dot / S) * s — kernels.c:71 / :126
template <int DT>
__device__ __forceinline__ float dequant_out(int dot, int asum, float s) {
  if (DT == 4) dot = (int)((unsigned)dot - 8u * (unsigned)asum);
  return fmul(div_qscale(dot, DT == 8), s);
}

// --------------------------------------------------------------------------
// activation truncation (kernels.c:66 / :113), once per row
// --------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) quantize_act_kernel(const float* __restrict__ x, int K,
                                                           uint8_t* __restrict__ act, int act_stride,
                                                           int* __restrict__ asum, int* err,
                                                           int mma_layout, int* flags, int mark) {
  const int m = blockIdx.x;
  const float* xr = x + (size_t)m * K;
  uint8_t* ar = act + (size_t)m * act_stride;
  int sum = 0, bad = 0;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const int a = trunc_scale(xr[k], DT == 8 ? 127.0f : 7.0f);
    if (DT == 8) {
      bad |= (a < -32768 || a > 32767);
      ar[k] = (uint8_t)(a & 0xFF);
      ar[K + k] = (uint8_t)((a >> 8) & 0xFF);
    } else {
      bad |= (a < -128 || a > 127);
      ar[mma_layout ? q4_mma_pos(k) : q4_act_pos(k)] = (uint8_t)(a & 0xFF);
      sum += a;
    }
  }
  if (bad) {
    if (mark) *err = mark;            // this call's mark (the GEMV compares it)
    else range_fail(err, flags, m);
  }
  if (DT == 4) {
    __shared__ int red[8];
    sum = warp_sum(sum);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
      int s = 0;
      for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
      asum[m] = s;
    }
  }
}

void launch_quantize_act(const float* x, int M, int K, int dtype, uint8_t* act, int act_stride,
                         int* asum, int* err, cudaStream_t st, int mma_layout, int* flags, int mark) {
  if (M <= 0) return;
  if (dtype == 2)
    quantize_act_kernel<8><<<M, 256, 0, st>>>(x, K, act, act_stride, asum, err, mma_layout, flags, mark);
  else
    quantize_act_kernel<4><<<M, 256, 0, st>>>(x, K, act, act_stride, asum, err, mma_layout, flags, mark);
}

// --------------------------------------------------------------------------
// sequential fp32 dot per output (test_model_trace.c:213-227, kernels.c:153-165)
// one dependent add chain per (m, n), exactly the reference's order
// --------------------------------------------------------------------------
template <bool VEC>
__global__ void __launch_bounds__(32) f32_seq_kernel(const float* __restrict__ A,
                                                     const float* __restrict__ W,
                                                     const float* __restrict__ b, float* __restrict__ C,
                                                     int M, int N, int K) {
  const long c = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= (long)M * N) return;
  const int m = (int)(c / N), n = (int)(c % N);
  const float* a = A + (size_t)m * K;
  const float* w = W + (size_t)n * K;
  float acc = 0.0f;
  if (VEC) {
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll 4
    for (int k = 0; k < K / 4; ++k) {
      const float4 av = __ldg(a4 + k), wv = __ldg(w4 + k);
      acc = fadd(acc, fmul(av.x, wv.x));
      acc = fadd(acc, fmul(av.y, wv.y));
      acc = fadd(acc, fmul(av.z, wv.z));
      acc = fadd(acc, fmul(av.w, wv.w));
    }
  } else {
    for (int k = 0; k < K; ++k) acc = fadd(acc, fmul(__ldg(a + k), __ldg(w + k)));
  }
  if (b) acc = fadd(acc, __ldg(b + n));   // logits += router_b (:466-468)
  C[c] = acc;
}

// Tiled form for the router: a CTA owns 16 experts x 16 tokens (one chain per
// thread); K is staged through shared memory in tiles of 256 with coalesced
// float4 loads, the next tile prefetched into registers while the current one
// is consumed. Each chain still adds its products one by one in k order.
constexpr int kRT = 16, kRE = 16, kRK = 128, kRPad = kRK + 4;

__global__ void __launch_bounds__(256) f32_seq_tiled_kernel(const float* __restrict__ A,
                                                           const float* __restrict__ W,
                                                           const float* __restrict__ b,
                                                           float* __restrict__ C, int M, int N,
                                                           int K) {
  __shared__ __align__(16) float xs[2][kRT][kRPad];
  __shared__ __align__(16) float ws[2][kRE][kRPad];
  const int tid = threadIdx.x;
  const int tt = tid / kRE, et = tid % kRE;
  const int m0 = blockIdx.y * kRT, n0 = blockIdx.x * kRE;
  // loader mapping: 16 rows x 32 float4 per tile; thread loads 2 float4 of each
  const int lrow = tid / 16, lcol = (tid % 16) * 2;   // 2 consecutive float4 per thread
  float4 rx[2], rw[2];
  auto gload = [&](int kt) {
    const int k0 = kt * kRK;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int kk = k0 + (lcol + i) * 4;
      const int m = m0 + lrow, n = n0 + lrow;
      rx[i] = (m < M && kk < K) ? __ldg(reinterpret_cast<const float4*>(A + (size_t)m * K + kk))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      rw[i] = (n < N && kk < K) ? __ldg(reinterpret_cast<const float4*>(W + (size_t)n * K + kk))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto sstore = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      *reinterpret_cast<float4*>(&xs[buf][lrow][(lcol + i) * 4]) = rx[i];
      *reinterpret_cast<float4*>(&ws[buf][lrow][(lcol + i) * 4]) = rw[i];
    }
  };
  const int ntiles = (K + kRK - 1) / kRK;
  float acc = 0.0f;
  gload(0);
  sstore(0);
  __syncthreads();
  for (int kt = 0; kt < ntiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ntiles) gload(kt + 1);
    const int kn = min(kRK, K - kt * kRK);
    const float* xr = xs[buf][tt];
    const float* wr = ws[buf][et];
    for (int k = 0; k < kn; k += 4) {
      const float4 xv = *reinterpret_cast<const float4*>(xr + k);
      const float4 wv = *reinterpret_cast<const float4*>(wr + k);
      acc = fadd(acc, fmul(xv.x, wv.x));
      acc = fadd(acc, fmul(xv.y, wv.y));
      acc = fadd(acc, fmul(xv.z, wv.z));
      acc = fadd(acc, fmul(xv.w, wv.w));
    }
    if (kt + 1 < ntiles) {
      sstore(buf ^ 1);
    }
    __syncthreads();
  }
  const int m = m0 + tt, n = n0 + et;
  if (m < M && n < N) {
    if (b) acc = fadd(acc, __ldg(b + n));
    C[(size_t)m * N + n] = acc;
  }
}

// Register-blocked form for many tokens (prefill): 128 threads; a thread
// owns TT tokens x ET experts of independent chains (instruction-level
// parallelism over dependent add chains); a CTA owns 8*TT tokens x 16*ET
// experts. k-tiles of 32 stream through an ST-deep shared-memory ring with
// 16-byte cp.async copies, ST-1 tiles in flight, so the load latency hides
// behind the chains of the tiles already there. A thread's experts are 16
// rows apart, so shared-memory reads hit distinct banks. Each output is still
// one sequential fp32 sum over k in ascending order.

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((unsigned)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int TT, int ET, int ST, int kGK>
__global__ void __launch_bounds__(128) f32_seq_gemm_kernel(const float* __restrict__ A,
                                                          const float* __restrict__ W,
                                                          const float* __restrict__ b,
                                                          float* __restrict__ C, int M, int N, int K) {
  constexpr int GT = 8 * TT, GE = 16 * ET, kGPad = kGK + 4;
  constexpr int CPR = kGK / 4;                           // 16-byte copies per row of a k-tile
  constexpr int XL = GT * CPR / 128, WL = GE * CPR / 128; // 16-byte copies per thread per k-tile
  extern __shared__ __align__(16) float smf[];
  float* xs = smf;                                        // [ST][GT][kGPad]
  float* ws = smf + ST * GT * kGPad;                      // [ST][GE][kGPad]
  const int tid = threadIdx.x;
  const int tq = tid / 16, eq = tid % 16;
  const int m0 = blockIdx.y * GT, n0 = blockIdx.x * GE;
  float acc[TT][ET];
#pragma unroll
  for (int i = 0; i < TT; ++i)
#pragma unroll
    for (int j = 0; j < ET; ++j) acc[i][j] = 0.0f;
  pdl_wait();
  pdl_launch();
  const int ntiles = (K + kGK - 1) / kGK;
  auto issue = [&](int kt) {
    const int sb = kt % ST, k0 = kt * kGK;
#pragma unroll
    for (int i = 0; i < XL; ++i) {
      const int q = tid + i * 128, row = q / CPR, col = (q % CPR) * 4;
      const int m = m0 + row;
      const bool v = m < M && k0 + col < K;
      cp_async16(&xs[((size_t)sb * GT + row) * kGPad + col], v ? A + (size_t)m * K + k0 + col : A, v ? 16 : 0);
    }
#pragma unroll
    for (int i = 0; i < WL; ++i) {
      const int q = tid + i * 128, row = q / CPR, col = (q % CPR) * 4;
      const int n = n0 + row;
      const bool v = n < N && k0 + col < K;
      cp_async16(&ws[((size_t)sb * GE + row) * kGPad + col], v ? W + (size_t)n * K + k0 + col : W, v ? 16 : 0);
    }
  };
#pragma unroll
  for (int st = 0; st < ST - 1; ++st) {
    if (st < ntiles) issue(st);
    cp_async_commit();
  }
  for (int kt = 0; kt < ntiles; ++kt) {
    cp_async_wait<ST - 2>();
    __syncthreads();          // tile kt landed for every thread; tile kt-1's stage is free
    if (kt + ST - 1 < ntiles) issue(kt + ST - 1);
    cp_async_commit();
    const int sb = kt % ST;
    const int kn = min(kGK, K - kt * kGK);
    const float* xb = xs + (size_t)sb * GT * kGPad;
    const float* wb = ws + (size_t)sb * GE * kGPad;
    // per 4 k: the next 4 k's shared loads first, then for each k all TT x ET
    // products before their TT x ET adds (inline PTX keeps this order; each
    // chain stays sequential in k)
    float4 xv[TT], wv[ET];
#pragma unroll
    for (int i = 0; i < TT; ++i) xv[i] = lds4(xb + (tq * TT + i) * kGPad);
#pragma unroll
    for (int j = 0; j < ET; ++j) wv[j] = lds4(wb + (eq + 16 * j) * kGPad);
#pragma unroll 2
    for (int k = 0; k < kn; k += 4) {
      const int kk = k + 4 < kn ? k + 4 : k;
      float4 xn[TT], wn[ET];
#pragma unroll
      for (int i = 0; i < TT; ++i) xn[i] = lds4(xb + (tq * TT + i) * kGPad + kk);
#pragma unroll
      for (int j = 0; j < ET; ++j) wn[j] = lds4(wb + (eq + 16 * j) * kGPad + kk);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float pr[TT][ET];
#pragma unroll
        for (int i = 0; i < TT; ++i) {
          const float xs = c == 0 ? xv[i].x : c == 1 ? xv[i].y : c == 2 ? xv[i].z : xv[i].w;
#pragma unroll
          for (int j = 0; j < ET; ++j)
            pr[i][j] = mul_rn(xs, c == 0 ? wv[j].x : c == 1 ? wv[j].y : c == 2 ? wv[j].z : wv[j].w);
        }
#pragma unroll
        for (int i = 0; i < TT; ++i)
#pragma unroll
          for (int j = 0; j < ET; ++j) acc[i][j] = add_rn(acc[i][j], pr[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TT; ++i) xv[i] = xn[i];
#pragma unroll
      for (int j = 0; j < ET; ++j) wv[j] = wn[j];
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < TT; ++i)
#pragma unroll
    for (int j = 0; j < ET; ++j) {
      const int m = m0 + tq * TT + i, n = n0 + eq + 16 * j;
      if (m < M && n < N) C[(size_t)m * N + n] = b ? fadd(acc[i][j], __ldg(b + n)) : acc[i][j];
    }
}

template <int TT, int ET, int ST, int GK>
static void launch_seq_gemm(dim3 grid, const float* A, const float* W, const float* b, float* C, int M, int N, int K,
                            cudaStream_t st) {
  const size_t smem = sizeof(float) * (size_t)ST * (8 * TT + 16 * ET) * (GK + 4);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(f32_seq_gemm_kernel<TT, ET, ST, GK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  launch_pdl(f32_seq_gemm_kernel<TT, ET, ST, GK>, grid, dim3(128), smem, st, A, W, b, C, M, N, K);
}

void launch_f32_seq_matmul(const float* A, const float* W, const float* b, float* C, int M, int N,
                           int K, cudaStream_t st) {
  const long total = (long)M * N;
  if (total <= 0) return;
  const bool aligned = ((uintptr_t)A % 16 == 0) && ((uintptr_t)W % 16 == 0);
  if (K % 4 == 0 && aligned && M >= 64) {
    // 4 x 4 chains per thread once there are enough tokens for a CTA per SM
    // (measured faster than 2 x 4 at two CTAs per SM); 2 x 2 below that, so
    // the grid still spreads over the SMs
    // (k-tile, stages) measured on Qwen3 router shapes (N=128, K=2048):
    // 4 x 4: (128, 3) 65.9 us at M=2048 against 78.3 with (32, 6);
    // 2 x 2: (256, 3) 30.2 us at M=512 against 33.2 with (128, 4)
    if (M >= 2048) {
      launch_seq_gemm<4, 4, 3, 128>(dim3((N + 63) / 64, (M + 31) / 32), A, W, b, C, M, N, K, st);
    } else {
      launch_seq_gemm<2, 2, 3, 256>(dim3((N + 31) / 32, (M + 15) / 16), A, W, b, C, M, N, K, st);
    }
    return;
  }
  if (K % 4 == 0 && aligned) {
    dim3 grid((N + kRE - 1) / kRE, (M + kRT - 1) / kRT);
    f32_seq_tiled_kernel<<<grid, 256, 0, st>>>(A, W, b, C, M, N, K);
    return;
  }
  const unsigned grid = (unsigned)((total + 31) / 32);
  f32_seq_kernel<false><<<grid, 32, 0, st>>>(A, W, b, C, M, N, K);
}

// --------------------------------------------------------------------------
// top-k (topk_desc, test_model_trace.c:275-288) + softmax (:481-487)
// --------------------------------------------------------------------------
constexpr int kMaxTopK = 32;

__global__ void topk_softmax_kernel(const float* __restrict__ logits, int T, int E, int K,
                                    int* __restrict__ idx, float* __restrict__ p) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float val[kMaxTopK];
  int id[kMaxTopK];
  for (int i = 0; i < K; ++i) { val[i] = -INFINITY; id[i] = -1; }
  const float* x = logits + (size_t)t * E;
  for (int e = 0; e < E; ++e) {
    const float v = x[e];
    int pos = -1;
    for (int i = 0; i < K; ++i) if (v > val[i]) { pos = i; break; }
    if (pos < 0) continue;
    for (int j = K - 1; j > pos; --j) { val[j] = val[j - 1]; id[j] = id[j - 1]; }
    val[pos] = v; id[pos] = e;
  }
  float mx = val[0];
  for (int i = 1; i < K; ++i) if (val[i] > mx) mx = val[i];
  float sum = 0.0f;
  for (int i = 0; i < K; ++i) { val[i] = exp_f32(__fsub_rn(val[i], mx)); sum = fadd(sum, val[i]); }
  const float inv = fdiv(1.0f, fadd(sum, 1e-9f));
  for (int i = 0; i < K; ++i) {
    idx[(size_t)t * K + i] = id[i];
    p[(size_t)t * K + i] = fmul(val[i], inv);
  }
}

// Warp per token: K rounds of a warp arg-max (larger value first, lower
// expert index on ties; NaN and -inf never chosen) — the same list topk_desc's
// insertion produces — then the softmax of :481-487 on lane 0.
constexpr int kTopkMaxPerLane = 8;   // E <= 256

__global__ void __launch_bounds__(256) topk_softmax_warp_kernel(const float* __restrict__ logits,
                                                               int T, int E, int K,
                                                               int* __restrict__ idx,
                                                               float* __restrict__ p) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float v[kTopkMaxPerLane];
  const float* x = logits + (size_t)t * E;
#pragma unroll
  for (int i = 0; i < kTopkMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? x[e] : -INFINITY;
  }
  float val[kMaxTopK];
  int id[kMaxTopK];
  for (int r = 0; r < K; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kTopkMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      if (v[i] > bv) { bv = v[i]; bi = e; }   // ascending e: first max kept
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const bool found = bi != 0x7fffffff;
    val[r] = found ? bv : -INFINITY;
    id[r] = found ? bi : -1;
    if (found && (bi & 31) == lane) {
#pragma unroll
      for (int i = 0; i < kTopkMaxPerLane; ++i)
        if (lane + 32 * i == bi) v[i] = -INFINITY;
    }
  }
  if (lane != 0) return;
  float mx = val[0];
  for (int i = 1; i < K; ++i) if (val[i] > mx) mx = val[i];
  float sum = 0.0f;
  for (int i = 0; i < K; ++i) { val[i] = exp_f32(__fsub_rn(val[i], mx)); sum = fadd(sum, val[i]); }
  const float inv = fdiv(1.0f, fadd(sum, 1e-9f));
  for (int i = 0; i < K; ++i) {
    idx[(size_t)t * K + i] = id[i];
    p[(size_t)t * K + i] = fmul(val[i], inv);
  }
}

void launch_topk_softmax(const float* logits, int T, int E, int K, int* idx, float* p,
                         cudaStream_t st) {
  if (T <= 0) return;
  if (E <= 32 * kTopkMaxPerLane) {
    topk_softmax_warp_kernel<<<(T + 7) / 8, 256, 0, st>>>(logits, T, E, K, idx, p);
  } else {
    topk_softmax_kernel<<<(T + 127) / 128, 128, 0, st>>>(logits, T, E, K, idx, p);
  }
}

// --------------------------------------------------------------------------
// routing lists: for every local expert with tokens, its slots (t*K+k) in
// ascending slot order; experts ascending. Optionally (nt > 0) also the tensor-
// core tile table (nt slots per tile) and the slot -> sorted-row map. One CTA;
// the token choices are staged in shared memory first.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) route_build_kernel(const int* __restrict__ idx, int TK,
                                                           int e_begin, int E_local, int* route,
                                                           int* hsum, int nt, int max_tiles,
                                                           int* slot_pos) {
  extern __shared__ int sm[];
  int* cnt = sm;                   // [E_local]
  int* start = sm + E_local;       // [E_local]
  int* sidx = sm + 2 * E_local;    // [TK]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const RouteView r = route_view(route, E_local);
  for (int i = threadIdx.x; i < TK; i += blockDim.x) {
    sidx[i] = idx[i];
    if (hsum) hsum[i] = 0;
  }
  __syncthreads();
  for (int el = wid; el < E_local; el += nw) {
    const int e = e_begin + el;
    int c = 0;
    for (int base = 0; base < TK; base += 32) {
      const int v = base + lane < TK ? sidx[base + lane] : -1;
      c += __popc(__ballot_sync(0xffffffffu, v == e));
    }
    if (lane == 0) cnt[el] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int na = 0, off = 0, ntl = 0;
    int* tab = route + 2 + 2 * E_local + TK;   // tile table: n | u[] | j0[] | cnt[]
    for (int el = 0; el < E_local; ++el) {
      start[el] = off;
      if (cnt[el] == 0) continue;
      r.active[na] = el;
      r.exp_off[na] = off;
      if (nt > 0)
        for (int j0 = off; j0 < off + cnt[el] && ntl < max_tiles; j0 += nt, ++ntl) {
          tab[1 + ntl] = na;
          tab[1 + max_tiles + ntl] = j0;
          tab[1 + 2 * max_tiles + ntl] = min(nt, off + cnt[el] - j0);
        }
      off += cnt[el];
      ++na;
    }
    r.exp_off[na] = off;
    *r.n_active = na;
    if (nt > 0) tab[0] = ntl;
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int el = wid; el < E_local; el += nw) {
    if (cnt[el] == 0) continue;
    const int e = e_begin + el;
    int pos = start[el];
    for (int base = 0; base < TK; base += 32) {
      const int v = base + lane < TK ? sidx[base + lane] : -1;
      const unsigned m = __ballot_sync(0xffffffffu, v == e);
      if (v == e) {
        const int j = pos + __popc(m & lt);
        r.slot_list[j] = base + lane;
        if (slot_pos) slot_pos[base + lane] = j;
      }
      pos += __popc(m);
    }
  }
}

int route_max_tiles(int TK, int E_local, int nt) {
  return TK / nt + (E_local < TK ? E_local : TK) + 1;
}

void launch_route_build(const int* idx, int T, int K, int e_begin, int e_end, int* route,
                        int E_local, int* hsum, int nt, int* slot_pos, cudaStream_t st) {
  (void)e_end;
  const int TK = T * K;
  const size_t smem = sizeof(int) * (2 * (size_t)E_local + (size_t)TK);
  const int mt = nt > 0 ? route_max_tiles(TK, E_local, nt) : 0;
  static size_t attr = 0;
  if (smem > 48 * 1024 && smem > attr) {
    cudaFuncSetAttribute(route_build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = smem;
  }
  // Plain launches for the prefill routing kernels (top-k, this, the
  // activation quantiser): chaining them with programmatic dependent launch
  // measured slower (Q4 T=2048 step 414 -> 450 us).
  route_build_kernel<<<1, 1024, smem, st>>>(idx, TK, e_begin, E_local, route, hsum, nt, mt, slot_pos);
}

// --------------------------------------------------------------------------
// routing lists for many slots (prefill), in one CTA of 1024 threads:
// per-expert counts by shared-memory atomics, one exclusive scan over the
// experts (warp shuffles; active list, offsets, tensor-core tile table), then
// each slot placed by a shared-memory atomic on its expert's fill counter.
// Slots land in arbitrary order within an expert; no result depends on it.
// --------------------------------------------------------------------------
constexpr int kRbMaxE = kRouteBuildMaxE;

__global__ void __launch_bounds__(1024) route_build_one_kernel(const int* __restrict__ idx, int TK, int e_begin,
                                                               int E_local, int* __restrict__ route,
                                                               int* __restrict__ hsum, int nt, int max_tiles,
                                                               int* __restrict__ slot_pos) {
  __shared__ int cnt[kRbMaxE], start[kRbMaxE], fill[kRbMaxE];
  __shared__ int s_wsum[3][kRbMaxE / 32];
  pdl_wait();
  pdl_launch();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < E_local; i += blockDim.x) { cnt[i] = 0; fill[i] = 0; }
  __syncthreads();
  for (int s = tid; s < TK; s += blockDim.x) {
    if (hsum) hsum[s] = 0;
    const int el = __ldg(idx + s) - e_begin;
    if (el >= 0 && el < E_local) atomicAdd(&cnt[el], 1);
  }
  __syncthreads();
  int* tab = route + 2 + 2 * E_local + TK;            // n_tiles | u[m] | j0[m] | cnt[m]
  const int mt = max_tiles;
  int xl = 0, xa = 0, xt = 0, c = 0, act = 0, til = 0;
  if (tid < kRbMaxE) {
    c = tid < E_local ? cnt[tid] : 0;
    act = c > 0;
    til = nt > 0 ? (c + nt - 1) / nt : 0;
    xl = c; xa = act; xt = til;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int yl = __shfl_up_sync(0xffffffffu, xl, o), ya = __shfl_up_sync(0xffffffffu, xa, o),
                yt = __shfl_up_sync(0xffffffffu, xt, o);
      if (lane >= o) { xl += yl; xa += ya; xt += yt; }
    }
    if (lane == 31) { s_wsum[0][warp] = xl; s_wsum[1][warp] = xa; s_wsum[2][warp] = xt; }
  }
  __syncthreads();
  if (tid < kRbMaxE) {
    for (int w = 0; w < warp; ++w) { xl += s_wsum[0][w]; xa += s_wsum[1][w]; xt += s_wsum[2][w]; }
    const int el = tid, off = xl - c, na = xa - act, ntl = xt - til;
    if (el < E_local) {
      start[el] = off;
      if (c > 0) {
        route[1 + na] = el;
        route[1 + E_local + na] = off;
        for (int j0 = off, k = ntl; nt > 0 && j0 < off + c && k < mt; j0 += nt, ++k) {
          tab[1 + k] = na;
          tab[1 + mt + k] = j0;
          tab[1 + 2 * mt + k] = min(nt, off + c - j0);
        }
      }
      if (el == E_local - 1) {
        route[1 + E_local + xa] = xl;                    // exp_off[n_active] = routed slots
        route[0] = xa;
        if (nt > 0) tab[0] = xt < mt ? xt : mt;
      }
    }
    if (E_local == 0 && tid == 0) { route[0] = 0; route[1] = 0; if (nt > 0) tab[0] = 0; }
  }
  __syncthreads();
  int* slots = route + 2 + 2 * E_local;
  for (int s = tid; s < TK; s += blockDim.x) {
    const int el = __ldg(idx + s) - e_begin;
    if (el < 0 || el >= E_local) continue;
    const int j = start[el] + atomicAdd(&fill[el], 1);
    slots[j] = s;
    if (slot_pos) slot_pos[s] = j;
  }
}

void launch_route_build_multi(const int* idx, int T, int K, int e_begin, int E_local, int* route, int* hsum,
                              int nt, int* slot_pos, cudaStream_t st) {
  const int TK = T * K;
  const int mt = nt > 0 ? route_max_tiles(TK, E_local, nt) : 0;
  launch_pdl(route_build_one_kernel, dim3(1), dim3(1024), 0, st, idx, TK, e_begin, E_local, route, hsum, nt, mt,
             slot_pos);
}

// --------------------------------------------------------------------------
// plain warp GEMV (matmul_f32_q8/_q4 fast path, and the batched C1 form)
// --------------------------------------------------------------------------
struct GemvArgs {
  const uint8_t* const* Wq;  // device array of n_mat pointers, or null
  const float* const* Ws;
  const uint8_t* W0;         // single matrix (when Wq == null)
  const float* S0;
  int n_mat, N, K, rb, cpl, np, items_per_mat, M, act_stride;
  const uint8_t* act;
  const int* asum;
  float* C;
  const float* A;            // fp32 activations [M][K], for the exact path
  const int* flag;           // == mark when the truncation kernel found an activation out of range
  int mark;
};

template <int DT>
__device__ __forceinline__ float exact_row(const float* __restrict__ a, const uint8_t* __restrict__ Wq,
                                           const float* __restrict__ Ws, int n, int K);

// the exact outputs of rows n0 .. n0+rows-1 of matrix `mat`, every m (kept
// out of line so the fast path's registers are unaffected)
template <int DT>
__device__ __noinline__ void gemv_exact_outputs(const float* A, float* C, const uint8_t* W, const float* S, int M,
                                                int N, int K, int n0, int rows) {
  for (int m = 0; m < M; ++m)
    for (int j = 0; j < rows; ++j)
      if (n0 + j < N) C[(size_t)m * N + n0 + j] = exact_row<DT>(A + (size_t)m * K, W, S, n0 + j, K);
}

template <int DT, int LPR, int RPG>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvArgs a) {
  constexpr int GPW = 32 / LPR;
  const int lane = threadIdx.x & 31, grp = lane / LPR, lig = lane % LPR;
  const long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int mat = (int)(w / a.items_per_mat);
  if (mat >= a.n_mat) return;
  const int item = (int)(w % a.items_per_mat);
  const uint8_t* W = a.Wq ? a.Wq[mat] : a.W0;
  const float* S = a.Ws ? a.Ws[mat] : a.S0;
  int n[RPG];
  bool ok[RPG];
#pragma unroll
  for (int j = 0; j < RPG; ++j) { n[j] = (item * GPW + grp) * RPG + j; ok[j] = n[j] < a.N; }
  if (a.flag && *a.flag == a.mark) {
    // an activation left the limb range: this warp's outputs are computed
    // exactly instead (int32 truncation, wrapping dot), one thread per output
    if (lig == 0) gemv_exact_outputs<DT>(a.A, a.C + (size_t)mat * a.M * a.N, W, S, a.M, a.N, a.K, n[0], RPG);
    return;
  }
  uint4 wr[RPG][4];
  auto load = [&](int p) {
#pragma unroll
    for (int j = 0; j < RPG; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = (p * a.cpl + i) * LPR + lig;
        wr[j][i] = (i < a.cpl && ok[j]) ? ldg_stream(W + (size_t)n[j] * a.rb + (size_t)c * 16)
                                        : make_uint4(0, 0, 0, 0);
      }
  };
  if (a.np == 1) load(0);
  for (int m = 0; m < a.M; ++m) {
    const uint8_t* act = a.act + (size_t)m * a.act_stride;
    int a0[RPG], a1[RPG];
#pragma unroll
    for (int j = 0; j < RPG; ++j) a0[j] = a1[j] = 0;
    for (int p = 0; p < a.np; ++p) {
      if (a.np > 1) load(p);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (i >= a.cpl) break;
        const int c = (p * a.cpl + i) * LPR + lig;
#pragma unroll
        for (int j = 0; j < RPG; ++j) chunk_dot<DT>(wr[j][i], act, a.K, c, a0[j], a1[j]);
      }
    }
    const int as = DT == 4 ? __ldg(a.asum + m) : 0;
#pragma unroll
    for (int j = 0; j < RPG; ++j) {
      const int v = group_sum<LPR>(lane_partial<DT>(a0[j], a1[j]));
      if (lig == 0 && ok[j])
        a.C[((size_t)mat * a.M + m) * a.N + n[j]] = dequant_out<DT>(v, as, __ldg(S + n[j]));
    }
  }
}

template <int DT, int RPG>
static void gemv_dispatch(const Geo& g, const GemvArgs& a, unsigned grid, cudaStream_t st) {
  switch (g.lpr) {
    case 1: gemv_kernel<DT, 1, RPG><<<grid, 256, 0, st>>>(a); break;
    case 2: gemv_kernel<DT, 2, RPG><<<grid, 256, 0, st>>>(a); break;
    case 4: gemv_kernel<DT, 4, RPG><<<grid, 256, 0, st>>>(a); break;
    case 8: gemv_kernel<DT, 8, RPG><<<grid, 256, 0, st>>>(a); break;
    case 16: gemv_kernel<DT, 16, RPG><<<grid, 256, 0, st>>>(a); break;
    default: gemv_kernel<DT, 32, RPG><<<grid, 256, 0, st>>>(a); break;
  }
}

bool launch_gemv(int dtype, const uint8_t* const* Wq, const float* const* Ws, int n_mat,
                 bool ptr_arrays_on_device, int N, int K, const uint8_t* act, int act_stride,
                 const int* asum, int M, float* C, cudaStream_t st, const float* A, const int* flag,
                 int mark) {
  Geo g;
  const int rb = dtype == 2 ? K : K / 2;
  if (dtype == 3 && (K & 1)) return false;
  if (!pick_geo(rb, g)) return false;
  constexpr int RPG = 2;
  GemvArgs a{};
  if (ptr_arrays_on_device) { a.Wq = Wq; a.Ws = Ws; }
  else { a.W0 = Wq[0]; a.S0 = Ws[0]; }
  a.n_mat = n_mat; a.N = N; a.K = K; a.rb = rb; a.cpl = g.cpl; a.np = g.np;
  const int rows_per_item = (32 / g.lpr) * RPG;
  a.items_per_mat = (N + rows_per_item - 1) / rows_per_item;
  a.M = M; a.act_stride = act_stride; a.act = act; a.asum = asum; a.C = C;
  a.A = A; a.flag = flag; a.mark = mark;
  const long warps = (long)a.items_per_mat * n_mat;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  if (dtype == 2) gemv_dispatch<8, RPG>(g, a, grid, st);
  else gemv_dispatch<4, RPG>(g, a, grid, st);
  return true;
}

// generic exact kernel for any shape / any activation magnitude: one thread
// per output, int32 activation, plain integer multiply-accumulate.
template <int DT>
__device__ __forceinline__ float exact_row(const float* __restrict__ a, const uint8_t* __restrict__ Wq,
                                           const float* __restrict__ Ws, int n, int K) {
  unsigned acc = 0;
  if (DT == 8) {
    const int8_t* w = reinterpret_cast<const int8_t*>(Wq) + (size_t)n * K;
    for (int k = 0; k < K; ++k) acc += (unsigned)(trunc_scale(__ldg(a + k), 127.0f) * (int)w[k]);
    return fmul(div_qscale((int)acc, true), __ldg(Ws + n));
  }
  const uint8_t* w = Wq + (size_t)n * (K / 2);
  for (int k = 0; k < K; k += 2) {
    const uint8_t b = w[k >> 1];
    acc += (unsigned)(trunc_scale(__ldg(a + k), 7.0f) * ((int)(b & 0xF) - 8));
    acc += (unsigned)(trunc_scale(__ldg(a + k + 1), 7.0f) * ((int)(b >> 4) - 8));
  }
  return fmul(div_qscale((int)acc, false), __ldg(Ws + n));
}

template <int DT>
__global__ void gemv_generic_kernel(const float* __restrict__ A, const uint8_t* __restrict__ Wq,
                                    const float* __restrict__ Ws, float* __restrict__ C, int M, int N, int K) {
  const long c = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= (long)M * N) return;
  const int m = (int)(c / N), n = (int)(c % N);
  C[c] = exact_row<DT>(A + (size_t)m * K, Wq, Ws, n, K);
}

void launch_gemv_generic(int dtype, const float* A, const uint8_t* Wq, const float* Ws, float* C,
                         int M, int N, int K, cudaStream_t st) {
  const long total = (long)M * N;
  if (total <= 0) return;
  const unsigned grid = (unsigned)((total + 127) / 128);
  if (dtype == 2) gemv_generic_kernel<8><<<grid, 128, 0, st>>>(A, Wq, Ws, C, M, N, K);
  else gemv_generic_kernel<4><<<grid, 128, 0, st>>>(A, Wq, Ws, C, M, N, K);
}

// --------------------------------------------------------------------------
// decode: fused gate/up GEMV + SiLU·up + re-truncation of h for the down
// projection (test_model_trace.c:496-501). One warp item = GPW row indices of
// one routed expert (each row index = one gate row and one up row), for every
// slot routed to that expert; weights are read once per item.
// --------------------------------------------------------------------------
struct GateUpArgs {
  const uint8_t* slab;
  size_t stride, gq_off, uq_off, gs_off, us_off;
  int F, D, rb, cpl, np, topk, items_per_expert;
  const int* route;  // n_active | active | exp_off | slot_list
  int E_local;
  const uint8_t* xact; int xact_stride;
  const int* xsum;
  uint8_t* hact; int hact_stride;
  int* hsum;
  int* err;
  int* flags;        // per-token range flags (range_fail) or null
};

template <int DT, int LPR>
__global__ void __launch_bounds__(256) gateup_kernel(const GateUpArgs a) {
  pdl_wait();
  pdl_launch();
  constexpr int GPW = 32 / LPR;
  constexpr float S = DT == 8 ? 127.0f : 7.0f;
  const int lane = threadIdx.x & 31, grp = lane / LPR, lig = lane % LPR;
  const long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const RouteView r = route_view(const_cast<int*>(a.route), a.E_local);
  const int u = (int)(w / a.items_per_expert);
  if (u >= *r.n_active) return;
  const int n = (int)(w % a.items_per_expert) * GPW + grp;
  const bool ok = n < a.F;
  const uint8_t* base = a.slab + (size_t)r.active[u] * a.stride;
  const uint8_t* Wg = base + a.gq_off + (size_t)n * a.rb;
  const uint8_t* Wu = base + a.uq_off + (size_t)n * a.rb;
  uint4 wg[4], wu[4];
  auto load = [&](int p) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = (p * a.cpl + i) * LPR + lig;
      const bool v = i < a.cpl && ok;
      wg[i] = v ? ldg_stream(Wg + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
      wu[i] = v ? ldg_stream(Wu + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
    }
  };
  if (a.np == 1) load(0);
  const float sg = ok ? __ldg(reinterpret_cast<const float*>(base + a.gs_off) + n) : 0.f;
  const float su = ok ? __ldg(reinterpret_cast<const float*>(base + a.us_off) + n) : 0.f;
  const int j0 = r.exp_off[u], j1 = r.exp_off[u + 1];
  for (int j = j0; j < j1; ++j) {
    const int s = r.slot_list[j];
    const int t = s / a.topk;
    const uint8_t* act = a.xact + (size_t)t * a.xact_stride;
    int g0 = 0, g1 = 0, u0 = 0, u1 = 0;
    for (int p = 0; p < a.np; ++p) {
      if (a.np > 1) load(p);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (i >= a.cpl) break;
        const int c = (p * a.cpl + i) * LPR + lig;
        chunk_dot<DT>(wg[i], act, a.D, c, g0, g1);
        chunk_dot<DT>(wu[i], act, a.D, c, u0, u1);
      }
    }
    const int dg = group_sum<LPR>(lane_partial<DT>(g0, g1));
    const int du = group_sum<LPR>(lane_partial<DT>(u0, u1));
    if (lig == 0 && ok) {
      const int as = DT == 4 ? __ldg(a.xsum + t) : 0;
      const float g = dequant_out<DT>(dg, as, sg);
      const float uu = dequant_out<DT>(du, as, su);
      const float h = fmul(silu_ref(g), uu);        // silu then g *= u (:498-501)
      const int ha = trunc_scale(h, S);             // down's activation truncation
      uint8_t* hr = a.hact + (size_t)s * a.hact_stride;
      if (DT == 8) {
        if (ha < -32768 || ha > 32767) range_fail(a.err, a.flags, t);
        hr[n] = (uint8_t)(ha & 0xFF);
        hr[a.F + n] = (uint8_t)((ha >> 8) & 0xFF);
      } else {
        if (ha < -128 || ha > 127) range_fail(a.err, a.flags, t);
        hr[q4_act_pos(n)] = (uint8_t)(ha & 0xFF);
        atomicAdd(a.hsum + s, ha);
      }
    }
  }
}

void launch_gateup(const LayerDev& L, const Workspace& ws, int T, int* err, cudaStream_t st) {
  Geo g;
  pick_geo(L.gu_rb, g);
  GateUpArgs a{};
  a.slab = L.slab; a.stride = L.expert_stride;
  a.gq_off = L.gq_off; a.uq_off = L.uq_off; a.gs_off = L.gs_off; a.us_off = L.us_off;
  a.F = L.F; a.D = L.D; a.rb = L.gu_rb; a.cpl = g.cpl; a.np = g.np; a.topk = L.topk;
  const int gpw = 32 / g.lpr;
  a.items_per_expert = (L.F + gpw - 1) / gpw;
  const int E_local = L.e_end - L.e_begin;
  a.route = ws.route; a.E_local = E_local;
  a.xact = ws.xact; a.xact_stride = 2 * L.D; a.xsum = ws.xsum;
  a.hact = ws.hact; a.hact_stride = 2 * L.F; a.hsum = ws.hsum; a.err = err;
  a.flags = ws.xbad;
  const int max_experts = E_local < T * L.topk ? E_local : T * L.topk;
  const long warps = (long)max_experts * a.items_per_expert;
  const unsigned grid = (unsigned)((warps + 7) / 8);
#define GU(DT)                                                                   \
  switch (g.lpr) {                                                               \
    case 1: launch_pdl(gateup_kernel<DT, 1>, dim3(grid), dim3(256), 0, st, a); break;                \
    case 2: launch_pdl(gateup_kernel<DT, 2>, dim3(grid), dim3(256), 0, st, a); break;                \
    case 4: launch_pdl(gateup_kernel<DT, 4>, dim3(grid), dim3(256), 0, st, a); break;                \
    case 8: launch_pdl(gateup_kernel<DT, 8>, dim3(grid), dim3(256), 0, st, a); break;                \
    case 16: launch_pdl(gateup_kernel<DT, 16>, dim3(grid), dim3(256), 0, st, a); break;              \
    default: launch_pdl(gateup_kernel<DT, 32>, dim3(grid), dim3(256), 0, st, a); break;              \
  }
  if (L.dtype == 2) { GU(8) } else { GU(4) }
#undef GU
}

// --------------------------------------------------------------------------
// decode: down projection (test_model_trace.c:502-503), slot rows y[s] for the
// k-ordered combine
// --------------------------------------------------------------------------
struct DownArgs {
  const uint8_t* slab;
  size_t stride, dq_off, ds_off;
  int D, F, rb, cpl, np, topk, items_per_expert, T;
  const int* route; int E_local;
  const uint8_t* hact; int hact_stride;
  const int* hsum;
  float* y;
};

template <int DT, int LPR, int RPG>
__global__ void __launch_bounds__(256) down_kernel(const DownArgs a) {
  pdl_wait();
  pdl_launch();
  constexpr int GPW = 32 / LPR;
  const int lane = threadIdx.x & 31, grp = lane / LPR, lig = lane % LPR;
  const long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const RouteView r = route_view(const_cast<int*>(a.route), a.E_local);
  const int na = *r.n_active;
  const int u = (int)(w / a.items_per_expert);
  if (u >= na) return;
  const int item = (int)(w % a.items_per_expert);
  const uint8_t* base = a.slab + (size_t)r.active[u] * a.stride;
  const uint8_t* W = base + a.dq_off;
  const float* S = reinterpret_cast<const float*>(base + a.ds_off);
  int n[RPG];
  bool ok[RPG];
  float sc[RPG];
#pragma unroll
  for (int j = 0; j < RPG; ++j) {
    n[j] = (item * GPW + grp) * RPG + j;
    ok[j] = n[j] < a.D;
    sc[j] = ok[j] ? __ldg(S + n[j]) : 0.f;
  }
  uint4 wr[RPG][4];
  auto load = [&](int p) {
#pragma unroll
    for (int j = 0; j < RPG; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = (p * a.cpl + i) * LPR + lig;
        wr[j][i] = (i < a.cpl && ok[j]) ? ldg_stream(W + (size_t)n[j] * a.rb + (size_t)c * 16)
                                        : make_uint4(0, 0, 0, 0);
      }
  };
  if (a.np == 1) load(0);
  const int j0 = r.exp_off[u], j1 = r.exp_off[u + 1];
  for (int jj = j0; jj < j1; ++jj) {
    const int s = r.slot_list[jj];
    const uint8_t* act = a.hact + (size_t)s * a.hact_stride;
    int a0[RPG], a1[RPG];
#pragma unroll
    for (int j = 0; j < RPG; ++j) a0[j] = a1[j] = 0;
    for (int p = 0; p < a.np; ++p) {
      if (a.np > 1) load(p);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (i >= a.cpl) break;
        const int c = (p * a.cpl + i) * LPR + lig;
#pragma unroll
        for (int j = 0; j < RPG; ++j) chunk_dot<DT>(wr[j][i], act, a.F, c, a0[j], a1[j]);
      }
    }
    const int as = DT == 4 ? __ldcg(a.hsum + s) : 0;
#pragma unroll
    for (int j = 0; j < RPG; ++j) {
      const int v = group_sum<LPR>(lane_partial<DT>(a0[j], a1[j]));
      if (lig == 0 && ok[j]) a.y[(size_t)s * a.D + n[j]] = dequant_out<DT>(v, as, sc[j]);
    }
  }
}

void launch_down(const LayerDev& L, const Workspace& ws, int T, float* y, cudaStream_t st) {
  Geo g;
  pick_geo(L.d_rb, g);
  constexpr int RPG = 2;
  DownArgs a{};
  a.slab = L.slab; a.stride = L.expert_stride; a.dq_off = L.dq_off; a.ds_off = L.ds_off;
  a.D = L.D; a.F = L.F; a.rb = L.d_rb; a.cpl = g.cpl; a.np = g.np; a.topk = L.topk; a.T = T;
  const int rows_per_item = (32 / g.lpr) * RPG;
  a.items_per_expert = (L.D + rows_per_item - 1) / rows_per_item;
  const int E_local = L.e_end - L.e_begin;
  a.route = ws.route; a.E_local = E_local;
  a.hact = ws.hact; a.hact_stride = 2 * L.F; a.hsum = ws.hsum;
  a.y = y;
  const int max_experts = E_local < T * L.topk ? E_local : T * L.topk;
  const long warps = (long)max_experts * a.items_per_expert;
  const unsigned grid = (unsigned)((warps + 7) / 8);
#define DN(DT)                                                                   \
  switch (g.lpr) {                                                               \
    case 1: launch_pdl(down_kernel<DT, 1, RPG>, dim3(grid), dim3(256), 0, st, a); break;             \
    case 2: launch_pdl(down_kernel<DT, 2, RPG>, dim3(grid), dim3(256), 0, st, a); break;             \
    case 4: launch_pdl(down_kernel<DT, 4, RPG>, dim3(grid), dim3(256), 0, st, a); break;             \
    case 8: launch_pdl(down_kernel<DT, 8, RPG>, dim3(grid), dim3(256), 0, st, a); break;             \
    case 16: launch_pdl(down_kernel<DT, 16, RPG>, dim3(grid), dim3(256), 0, st, a); break;           \
    default: launch_pdl(down_kernel<DT, 32, RPG>, dim3(grid), dim3(256), 0, st, a); break;           \
  }
  if (L.dtype == 2) { DN(8) } else { DN(4) }
#undef DN
}

// k-ordered combine + residual as a separate pass (prefill, expert parallel)
// out[t] = xres[t] + Σ_k p[t][k] y[t*K+k] in k order (test_model_trace.c:513,
// :517), or with seq_residual out[t] = (xres[t] + p0 y0) + p1 y1 ... as
// model.c:188 accumulates into x directly. A slot with no expert (idx < 0:
// fewer than K logits that are neither NaN nor -inf) adds p * 0: the
// reference reads an expert out of bounds there, and its p is 0 (finite
// maximum) or NaN (no finite logit), which gives 0 or NaN whatever that
// expert holds. idx may be null (every slot has an expert).
__global__ void combine_kernel(const float* __restrict__ y, const float* __restrict__ p,
                               const int* __restrict__ idx, const float* xres, float* out, int T, int D, int K,
                               int seq, const HostOut ho) {
  pdl_wait();
  pdl_launch();
  const long q = (long)blockIdx.x * blockDim.x + threadIdx.x;
  publish_host(ho, q, (long)gridDim.x * blockDim.x);
  if (q >= (long)T * D) return;
  const int t = (int)(q / D), n = (int)(q % D);
  float acc = seq ? xres[q] : 0.0f;
  for (int k = 0; k < K; ++k) {
    const int s = t * K + k;
    const float yv = (idx && idx[s] < 0) ? 0.0f : y[(size_t)s * D + n];
    acc = fadd(acc, fmul(p[s], yv));
  }
  out[q] = seq ? acc : fadd(xres[q], acc);
}

void launch_combine(const float* y, const float* p, const int* idx, const float* xres, float* out, int T, int D,
                    int K, cudaStream_t st, bool seq_residual, const HostOut& ho) {
  const long total = (long)T * D;
  if (total <= 0) return;
  launch_pdl(combine_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, y, p, idx, xres, out, T, D,
             K, seq_residual ? 1 : 0, ho);
}

// --------------------------------------------------------------------------
// rowwise quantisers, export.py:23-36 (bit-exact): s = max(amax,1e-8)/127 or
// /7 in fp32; q = round-half-even(w / s) (Q4: clamp [-8,7], +8, pack pairs)
// --------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) quantize_rowwise_kernel(const float* __restrict__ W,
                                                               int cols, void* q, float* s) {
  const int r = blockIdx.x;
  const float* w = W + (size_t)r * cols;
  float amax = 0.0f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) amax = fmaxf(amax, fabsf(w[c]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
    red[0] = fdiv(fmaxf(m, 1e-8f), DT == 8 ? 127.0f : 7.0f);
  }
  __syncthreads();
  const float sc = red[0];
  if (threadIdx.x == 0) s[r] = sc;
  if (DT == 8) {
    int8_t* qr = reinterpret_cast<int8_t*>(q) + (size_t)r * cols;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) qr[c] = (int8_t)__float2int_rn(fdiv(w[c], sc));
  } else {
    uint8_t* qr = reinterpret_cast<uint8_t*>(q) + (size_t)r * (cols / 2);
    for (int c = threadIdx.x; c < cols / 2; c += blockDim.x) {
      int v0 = __float2int_rn(fdiv(w[2 * c], sc)), v1 = __float2int_rn(fdiv(w[2 * c + 1], sc));
      v0 = min(max(v0, -8), 7) + 8;
      v1 = min(max(v1, -8), 7) + 8;
      qr[c] = (uint8_t)(v0 | (v1 << 4));
    }
  }
}

void launch_quantize_rowwise(int dtype, const float* W, int rows, int cols, void* q, float* s,
                             cudaStream_t st) {
  if (rows <= 0) return;
  if (dtype == 2) quantize_rowwise_kernel<8><<<rows, 256, 0, st>>>(W, cols, q, s);
  else quantize_rowwise_kernel<4><<<rows, 256, 0, st>>>(W, cols, q, s);
}

// --------------------------------------------------------------------------
// synthetic N(0, std²): sample i = Box-Muller of outputs 2i, 2i+1 of
// splitmix64 seeded with `seed`, in double, rounded once to float
// --------------------------------------------------------------------------
__device__ inline uint64_t splitmix_at(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void synth_normal_kernel(uint64_t seed, uint64_t offset, size_t n, float std, float* out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t j = offset + i;
  const double u1 = (double)(splitmix_at(seed, 2 * j) >> 11) * 0x1.0p-53;
  const double u2 = (double)(splitmix_at(seed, 2 * j + 1) >> 11) * 0x1.0p-53;
  const double z = sqrt(-2.0 * log(1.0 - u1)) * cos(6.283185307179586 * u2);
  out[i] = (float)(z * (double)std);
}

void launch_synth_normal(uint64_t seed, uint64_t offset, size_t n, float std, float* out,
                         cudaStream_t st) {
  if (!n) return;
  synth_normal_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(seed, offset, n, std, out);
}

__global__ void zero_kernel(float* C, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) C[i] = 0.0f;
}
void launch_zero_fill(float* C, size_t n, cudaStream_t st) {
  if (!n) return;
  zero_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(C, n);
}

}  // namespace moe
