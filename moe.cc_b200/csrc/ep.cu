// ep.cu — expert parallelism with the slot exchange fused into the down GEMM.
//
// Every rank routes all T*N tokens (identical results) and computes its own
// experts' slots. The down projection's epilogue (moe_mma.cu, ep mode) stores
// each slot's output row directly into the receive buffer of the rank that
// owns the slot's token, over NVLink (plain peer stores; peer buffers opened
// through CUDA IPC). Then:
//   ep_signal_kernel   raises this rank's flag at every peer (system-scope
//                      release after a system fence), value = call sequence
//   ep_combine_kernel  waits (bounded) until every rank's flag reached the
//                      sequence, then applies the k-ordered combine + residual
//                      (test_model_trace.c:513,517) to this rank's tokens.
// Exactly one rank writes each slot row, so no reduction is involved. The
// flags only ever grow, so they need no reset between calls. The wait gives
// up after kWaitBudget polls and reports kErrTimeout instead of hanging.
// Requires one GPU per rank: a kernel waiting on another rank never shares a
// GPU with that rank's kernels.
#include "common.cuh"
#include "kernels.cuh"
#include "pipeline.cuh"

namespace moe {

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void ep_signal_kernel(unsigned long long* const* peer_flags, int rank, int world,
                                 unsigned long long seq) {
  const int p = threadIdx.x;
  if (p >= world) return;
  __threadfence_system();
  st_release_sys(peer_flags[p] + rank, seq);
}

__global__ void __launch_bounds__(256) ep_combine_kernel(const unsigned long long* flags, int world,
                                                         unsigned long long seq, const float* __restrict__ y,
                                                         const float* __restrict__ p, const int* __restrict__ idx,
                                                         const float* xres, float* out, int T, int D, int K,
                                                         int* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int src = 0; src < world && ok; ++src) {
      uint32_t i = 0;
      while (ld_acquire_sys(flags + src) < seq)
        if (++i >= kWaitBudget) { ok = 0; break; }
    }
    if (!ok) atomicOr(err, kErrTimeout);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const long q = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= (long)T * D) return;
  const int t = (int)(q / D), n = (int)(q % D);
  float acc = 0.0f;
  for (int k = 0; k < K; ++k) {
    const int s = t * K + k;
    if (idx[s] < 0) continue;
    acc = fadd(acc, fmul(p[s], __ldcg(y + (size_t)s * D + n)));
  }
  out[q] = fadd(xres[q], acc);
}

void launch_ep_signal(unsigned long long* const* peer_flags, int rank, int world, unsigned long long seq,
                      cudaStream_t st) {
  ep_signal_kernel<<<1, 32, 0, st>>>(peer_flags, rank, world, seq);
}

void launch_ep_combine(const unsigned long long* flags, int world, unsigned long long seq, const float* y,
                       const float* p, const int* idx, const float* xres, float* out, int T, int D, int K,
                       int* err, cudaStream_t st) {
  const long total = (long)T * D;
  if (total <= 0) return;
  ep_combine_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(flags, world, seq, y, p, idx, xres,
                                                                       out, T, D, K, err);
}

}  // namespace moe
