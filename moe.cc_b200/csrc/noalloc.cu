// noalloc.cu — moe_matmul_q_dev_noalloc: the Q8/Q4 device matmul for callers
// that cannot allocate GPU memory.
//
// Some hosts cannot call cudaMalloc at the point where they need a matmul:
// code running inside a custom allocator or a memory-pool callback, embedders
// whose GPU memory is fully pre-reserved by a framework, or real-time paths
// where an allocation's implicit synchronisation is not allowed. The regular
// moe_matmul_q8_dev/_q4_dev grow a private scratch buffer with cudaMalloc on
// first use; this variant keeps its scratch in a fixed file-scope device
// array instead and never allocates.
//
// Scratch: one static array of kNoAllocBytes per GPU that loads the library
// (held until the process exits): an error word, the per-row activation sums
// (at most kMaxRows rows) and the truncated activation planes (2 bytes per
// element, at most kMaxPlaneBytes, i.e. M*K <= 524288).
// All calls share the array and it keeps the previous call's contents; the
// error word is cleared at the start of each call. Calls whose GPU work
// overlaps (different streams, no ordering between them) race on the array.
// The first call on each device looks up the array's device address
// (cudaGetSymbolAddress) with that device current; make that first call
// before any stream capture.
#include <cuda_runtime.h>
#include <stdio.h>

#include "../../include/moe_cuda.h"
#include "common.cuh"
#include "kernels.cuh"

namespace moe {

int set_error_message(int code, const char* msg);   // runtime.cu

namespace na {

constexpr int kMaxRows = 4096;
constexpr size_t kHeaderBytes = 256;                                 // error word
constexpr size_t kSumBytes = sizeof(int) * kMaxRows;                 // 16 KiB
constexpr size_t kMaxPlaneBytes = 1u << 20;                          // 1 MiB
constexpr size_t kNoAllocBytes = kHeaderBytes + kSumBytes + kMaxPlaneBytes;

static __device__ __align__(256) uint8_t g_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
static uint8_t* g_addr[kMaxDevices];   // device address of g_scratch, per device

// Exact int32 recomputation of C, run only when the truncation kernel flagged
// an activation outside the fast path's limb range (same arithmetic as
// kernels.c:51-128: truncation, wrapping int32 dot, IEEE divide and multiply).
template <int DT>
__global__ void exact_fixup_kernel(const int* __restrict__ flag, const float* __restrict__ A,
                                   const uint8_t* __restrict__ Wq, const float* __restrict__ Ws,
                                   float* __restrict__ C, int M, int N, int K) {
  if (*flag == 0) return;
  const long c = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= (long)M * N) return;
  const int m = (int)(c / N), n = (int)(c % N);
  const float* a = A + (size_t)m * K;
  unsigned acc = 0;
  if (DT == 8) {
    const int8_t* w = reinterpret_cast<const int8_t*>(Wq) + (size_t)n * K;
    for (int k = 0; k < K; ++k) acc += (unsigned)(trunc_scale(a[k], 127.0f) * (int)w[k]);
    C[c] = fmul(div_qscale((int)acc, true), Ws[n]);
  } else {
    const uint8_t* w = Wq + (size_t)n * (K / 2);
    for (int k = 0; k < K; k += 2) {
      const uint8_t b = w[k >> 1];
      acc += (unsigned)(trunc_scale(a[k], 7.0f) * ((int)(b & 0xF) - 8));
      acc += (unsigned)(trunc_scale(a[k + 1], 7.0f) * ((int)(b >> 4) - 8));
    }
    C[c] = fmul(div_qscale((int)acc, false), Ws[n]);
  }
}

static uint8_t* scratch_address(int* rc) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *rc = set_error_message(MOE_ERR_CUDA, "moe_matmul_q_dev_noalloc: no usable current device");
    return nullptr;
  }
  if (!g_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p) {
      char msg[256];
      snprintf(msg, sizeof(msg), "moe_matmul_q_dev_noalloc: cudaGetSymbolAddress failed: %s",
               cudaGetErrorString(e));
      *rc = set_error_message(MOE_ERR_CUDA, msg);
      return nullptr;
    }
    g_addr[dev] = static_cast<uint8_t*>(p);
  }
  return g_addr[dev];
}

}  // namespace na
}  // namespace moe

using namespace moe;

extern "C" int moe_matmul_q_dev_noalloc(const float* A, const void* B_q, const float* B_s, float* C,
                                        int M, int N, int K, int dtype, void* stream) {
  char msg[256];
  if (dtype != MOE_DTYPE_Q8 && dtype != MOE_DTYPE_Q4)
    return set_error_message(MOE_ERR_INVALID, "moe_matmul_q_dev_noalloc: dtype must be 2 (Q8) or 3 (Q4)");
  if (M < 0 || N < 0 || K < 0)
    return set_error_message(MOE_ERR_INVALID, "moe_matmul_q_dev_noalloc: negative M/N/K");
  if (dtype == MOE_DTYPE_Q4 && (K & 1))
    return set_error_message(MOE_ERR_UNSUPPORTED, "moe_matmul_q_dev_noalloc: Q4 needs an even K");
  if (M > na::kMaxRows || (size_t)2 * M * K > na::kMaxPlaneBytes) {
    snprintf(msg, sizeof(msg),
             "moe_matmul_q_dev_noalloc: M=%d K=%d exceeds the fixed scratch (M <= %d and M*K <= %zu)",
             M, K, na::kMaxRows, na::kMaxPlaneBytes / 2);
    return set_error_message(MOE_ERR_INVALID, msg);
  }
  if ((long)M * N == 0) return MOE_OK;
  int rc = MOE_OK;
  uint8_t* base = na::scratch_address(&rc);
  if (!base) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  int* flag = reinterpret_cast<int*>(base);
  int* asum = reinterpret_cast<int*>(base + na::kHeaderBytes);
  uint8_t* act = base + na::kHeaderBytes + na::kSumBytes;
  const unsigned grid = (unsigned)(((long)M * N + 127) / 128);
  cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), st);
  if (e == cudaSuccess) {
    if (K > 0 && ((uintptr_t)B_q % 16 == 0) && fast_geometry_ok(dtype, K)) {
      // truncated activation planes in the static array, then the warp GEMV;
      // the fix-up pass recomputes C exactly if any activation was out of range
      launch_quantize_act(A, M, K, dtype, act, 2 * K, asum, flag, st);
      const uint8_t* wq = static_cast<const uint8_t*>(B_q);
      launch_gemv(dtype, &wq, &B_s, 1, false, N, K, act, 2 * K, asum, M, C, st);
      if (dtype == MOE_DTYPE_Q8)
        na::exact_fixup_kernel<8><<<grid, 128, 0, st>>>(flag, A, wq, B_s, C, M, N, K);
      else
        na::exact_fixup_kernel<4><<<grid, 128, 0, st>>>(flag, A, wq, B_s, C, M, N, K);
    } else {
      // shapes without a fast geometry need no scratch: exact kernel directly
      launch_gemv_generic(dtype, A, static_cast<const uint8_t*>(B_q), B_s, C, M, N, K, st);
    }
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "moe_matmul_q_dev_noalloc: %s", cudaGetErrorString(e));
    return set_error_message(MOE_ERR_CUDA, msg);
  }
  return MOE_OK;
}
