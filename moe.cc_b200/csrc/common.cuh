// common.cuh — shared device helpers for libmoe_cuda (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <utility>

#include "expf_ref.h"

namespace moe {

// Exactly-rounded scalar ops used wherever the reference's arithmetic must be
// reproduced bit for bit (no FMA contraction, IEEE round-to-nearest).
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// expf with the C library's results, bit for bit (expf_ref.h): the softmax
// and SiLU exponentials of the reference (test_model_trace.c:233,485).
__device__ __forceinline__ float exp_f32(float v) { return expf_ref(v); }

// silu_f32 (test_model_trace.c:229-236): v / (1 + expf(-v)).
__device__ __forceinline__ float silu_ref(float v) {
  return fdiv(v, fadd(1.0f, exp_f32(-v)));
}

// Inline-PTX forms of the exact multiply and add and of a 16-byte shared
// load, for the sequential fp32 chains: the compiler keeps asm statements in
// the order written, so a chain loop can issue a block's products and the next
// block's loads before the block's dependent adds (from plain C++ the loads
// sank next to their uses and each add waited on its own multiply: the routing
// chains measured 6.6 against 4.9 cycles per add). mul.rn / add.rn are IEEE
// single with no contraction, as __fmul_rn / __fadd_rn.
__device__ __forceinline__ float4 lds4(const float* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"((unsigned)__cvta_generic_to_shared(p)));
  return v;
}
__device__ __forceinline__ float mul_rn(float a, float b) {
  float r;
  asm volatile("mul.rn.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float add_rn(float a, float b) {
  float r;
  asm volatile("add.rn.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// (float)d / S, IEEE round-to-nearest, for an int32 d and the quantisation
// divisors S = 127 (Q8) and 7 (Q4), as the reference's ((float)dot / 127f)
// (kernels.c:71 / :126). Markstein's correction of the reciprocal product: with
// r = RN(1/S), q0 = RN(x r), the remainder x - q0 S is exact under FMA and
// RN(q0 + rem r) is the correctly rounded quotient. Checked against IEEE
// division for every one of the 2^32 inputs and both divisors
// (tests/divide_check.c). One multiply and two FMAs instead of a divide.
__device__ __forceinline__ float div_qscale(int d, bool q8) {
  const float S = q8 ? 127.0f : 7.0f;
  const float r = q8 ? 0x1.020408p-7f : 0x1.24924ap-3f;   // RN(1/127), RN(1/7)
  const float x = __int2float_rn(d);
  const float q0 = __fmul_rn(x, r);
  return __fmaf_rn(__fmaf_rn(-q0, S, x), r, q0);
}

// (int32_t)(a * scale) — kernels.c:66 / :113, truncation toward zero.
// Returns INT32_MIN for NaN, infinities and |v| >= 2^31: the reference's
// x86-64 build converts with cvttss2si, which gives that "indefinite" value
// for every input outside the int32 range (the GPU's conversion saturates).
__device__ __forceinline__ int trunc_scale(float a, float scale) {
  float v = fmul(a, scale);
  if (!(fabsf(v) < 2147483648.0f)) return INT32_MIN;
  return __float2int_rz(v);
}

// dp4a with signed A bytes and unsigned B bytes: d = c + Σ a_i * b_i.
__device__ __forceinline__ int dp4a_su(int a, unsigned b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// signed × signed
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }
// unsigned A × signed B (int8 weights against the low activation limb)
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 16-byte read-only streaming load (weights: read once, keep out of L1).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Q8 activation limbs: a = lo + 256 * hi with lo in [0,255], hi in [-128,127]
// (|a| <= 32767). Σ w*a = Σ w*lo + 256 Σ w*hi, exact mod 2^32.
// Q8 chunk dot: 16 weight bytes against 16 lo bytes and 16 hi bytes.
__device__ __forceinline__ void dot16_q8(const uint4 w, const uint4 lo, const uint4 hi,
                                         int& acc_lo, int& acc_hi) {
  acc_lo = dp4a_us(lo.x, (int)w.x, acc_lo);
  acc_lo = dp4a_us(lo.y, (int)w.y, acc_lo);
  acc_lo = dp4a_us(lo.z, (int)w.z, acc_lo);
  acc_lo = dp4a_us(lo.w, (int)w.w, acc_lo);
  acc_hi = dp4a_ss((int)hi.x, (int)w.x, acc_hi);
  acc_hi = dp4a_ss((int)hi.y, (int)w.y, acc_hi);
  acc_hi = dp4a_ss((int)hi.z, (int)w.z, acc_hi);
  acc_hi = dp4a_ss((int)hi.w, (int)w.w, acc_hi);
}

// Q4 chunk dot: 16 packed bytes (32 nibbles, k = 32c..32c+31) against 32
// signed activation bytes stored as words [E0,O0,E1,O1] [E2,O2,E3,O3], where
// word j of the weights holds k=8j..8j+7 with even k in low nibbles:
// Ej = (a[8j],a[8j+2],a[8j+4],a[8j+6]), Oj = (a[8j+1],a[8j+3],a[8j+5],a[8j+7]).
// Accumulates Σ a * nibble (nibble in [0,15]); the caller subtracts 8 Σ a.
__device__ __forceinline__ int dot16_q4(const uint4 w, const uint4 a0, const uint4 a1, int acc) {
  acc = dp4a_su((int)a0.x, w.x & 0x0F0F0F0Fu, acc);
  acc = dp4a_su((int)a0.y, (w.x >> 4) & 0x0F0F0F0Fu, acc);
  acc = dp4a_su((int)a0.z, w.y & 0x0F0F0F0Fu, acc);
  acc = dp4a_su((int)a0.w, (w.y >> 4) & 0x0F0F0F0Fu, acc);
  acc = dp4a_su((int)a1.x, w.z & 0x0F0F0F0Fu, acc);
  acc = dp4a_su((int)a1.y, (w.z >> 4) & 0x0F0F0F0Fu, acc);
  acc = dp4a_su((int)a1.z, w.w & 0x0F0F0F0Fu, acc);
  acc = dp4a_su((int)a1.w, (w.w >> 4) & 0x0F0F0F0Fu, acc);
  return acc;
}

// Position of activation element k inside the Q4 permuted layout
// (byte offset within the token's row of K bytes).
__host__ __device__ __forceinline__ int q4_act_pos(int k) {
  const int j = k >> 3, r = k & 7;           // word j of weights, nibble r
  return (j << 3) + ((r & 1) << 2) + (r >> 1);  // E_j at 8j..8j+3, O_j at 8j+4..
}

// Position of activation element k in the tensor-core Q4 layout: within each
// 32-element group, the even elements first, then the odd ones. This matches
// how the tensor-core path unpacks 16 packed weight bytes (32 nibbles) into 16
// low-nibble bytes followed by 16 high-nibble bytes.
__host__ __device__ __forceinline__ int q4_mma_pos(int k) {
  return (k & ~31) + ((k & 1) << 4) + ((k & 31) >> 1);
}

// ---- programmatic dependent launch ----------------------------------------
// The kernels of one MoE call are launched with programmatic stream
// serialization: a kernel may start while its predecessor in the stream still
// runs. Each kernel runs pdl_wait() before it touches anything the
// predecessor writes or reads, and signals pdl_launch() only after its own
// pdl_wait(), so when a kernel starts, everything two launches back is
// complete. Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with programmatic stream serialization (MOE_PDL=0 turns it off).
bool pdl_enabled();
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid; cfg.blockDim = block; cfg.dynamicSmemBytes = smem; cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---- optional step timeline (build with -DMOE_TIMELINE) ---------------------
// Each hooked kernel records the globaltimer of its first CTA start and last
// CTA end (ns) in a device table, read by moe_debug_timeline(). Without the
// macro the hooks compile to nothing.
enum : int { kTlRoute = 0, kTlGather, kTlGateup, kTlDown, kTlCombine, kTlCount };
#ifdef MOE_TIMELINE
// one table per translation unit (no relocatable device code); each file
// that launches hooked kernels ends with MOE_TL_IO(name), and the runtime
// merges the tables
static __device__ unsigned long long g_timeline[kTlCount][2];
#define MOE_TL_IO(name)                                                              \
  void tl_io_##name(unsigned long long* out, int reset) {                           \
    unsigned long long t[kTlCount][2];                                              \
    cudaMemcpyFromSymbol(t, g_timeline, sizeof(t));                                 \
    for (int i = 0; i < kTlCount; ++i) {                                            \
      if (t[i][0] < out[2 * i]) out[2 * i] = t[i][0];                               \
      if (t[i][1] > out[2 * i + 1]) out[2 * i + 1] = t[i][1];                       \
      t[i][0] = ~0ull; t[i][1] = 0;                                                 \
    }                                                                               \
    if (reset) cudaMemcpyToSymbol(g_timeline, t, sizeof(t));                        \
  }
__device__ __forceinline__ unsigned long long tl_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#define MOE_TL_START(id) do { if (threadIdx.x == 0) atomicMin(&::moe::g_timeline[id][0], ::moe::tl_now()); } while (0)
#define MOE_TL_END(id) do { if (threadIdx.x == 0) atomicMax(&::moe::g_timeline[id][1], ::moe::tl_now()); } while (0)
#else
#define MOE_TL_IO(name)
#define MOE_TL_START(id) do { } while (0)
#define MOE_TL_END(id) do { } while (0)
#endif

// Error flag bits written by kernels (read by the host).
enum : int { kErrRange = 1, kErrTimeout = 2 };

// Records an activation of token t outside the fast kernels' integer range
// (or NaN/inf). With per-call token flags (moe_ffn: flags[0] = any token,
// flags[1] = arrival counter of the fix-up pass, flags[2 + t] = token t) the
// exact fix-up pass recomputes that token's slots; without them the call's
// error word gets kErrRange.
__device__ __forceinline__ void range_fail(int* err, int* flags, int t) {
  if (flags) { flags[2 + t] = 1; flags[0] = 1; }
  else atomicOr(err, kErrRange);
}

}  // namespace moe
