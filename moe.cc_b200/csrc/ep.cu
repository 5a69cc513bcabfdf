// ep.cu — the combine of the expert-parallel exchange.
//
// Every rank routes its own tokens and sends their activations and top-k to
// every rank (router.cu, EP mode); each rank computes its own experts' slots,
// and the down projection's epilogue stores each slot row straight into the
// y buffer of the rank owning the slot's token, over NVLink (moe_mma.cu, EP
// mode), whose last CTA raises this rank's combine flag at every peer.
// ep_combine_kernel waits (bounded) until every rank's combine flag reached
// this call's sequence number and applies the k-ordered combine + residual
// (test_model_trace.c:513,517) to this rank's tokens. Exactly one rank writes
// each slot row, so no reduction is involved. The wait gives up after the
// group's time limit (EpView::wait_ns) and reports kErrTimeout instead of
// hanging.
// Requires one GPU per rank: a kernel waiting on another rank never shares a
// GPU with that rank's kernels.
#include "common.cuh"
#include "kernels.cuh"
#include "pipeline.cuh"

namespace moe {

__global__ void __launch_bounds__(256) ep_combine_kernel(const EpView ep, const float* xres, float* out,
                                                         int D, int K, int* err) {
  __shared__ int s_ok;
  MOE_TL_START(kTlCombine);
  pdl_wait();
  pdl_launch();
  const uint8_t* mine = ep.base_local;
  if (threadIdx.x == 0) {
    const int ok = wait_flags_sys(reinterpret_cast<const unsigned long long*>(mine + kEpCombineFlags),
                                  ep.world, ep.seq, ep.wait_ns);
    if (!ok) atomicOr(err, kErrTimeout);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int T = ep.T_local;
  const long q = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= (long)T * D) return;
  const int t = (int)(q / D), n = (int)(q % D);
  const size_t s0 = (size_t)ep.rank * T * K;                   // this rank's first slot
  const float* p = reinterpret_cast<const float*>(mine + ep.p_off) + s0;
  const float* y = reinterpret_cast<const float*>(mine + ep.y_off);
  float acc = 0.0f;
  for (int k = 0; k < K; ++k) {
    const int s = t * K + k;
    acc = fadd(acc, fmul(__ldcg(p + s), __ldcg(y + (size_t)s * D + n)));
  }
  out[q] = fadd(xres[q], acc);
  MOE_TL_END(kTlCombine);
}

void launch_ep_combine(const EpView& ep, const float* xres, float* out, int D, int K, int* err,
                       cudaStream_t st) {
  const long total = (long)ep.T_local * D;
  if (total <= 0) return;
  launch_pdl(ep_combine_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, ep, xres, out, D, K, err);
}

MOE_TL_IO(ep)

}  // namespace moe
