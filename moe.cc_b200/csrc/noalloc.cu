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
// Only shapes that take the fast path use the array (K a multiple of 16 bytes
// of packed row, 16-byte aligned B_q); the limits apply to those shapes, the
// others run the exact kernel directly and have none.
// All calls share the array and it keeps the previous call's contents; the
// error word holds the mark of the last call that found an activation out of
// range (each call compares its own mark). Calls whose GPU work
// overlaps (different streams, no ordering between them) race on the array.
// The first call on each device is the set-up: with that device current it
// looks up the array's device address (cudaGetSymbolAddress) and keeps it.
// With CUDA's lazy module loading that first call also loads the library's
// kernels onto the device, which allocates device memory; make it before any
// stream capture and outside any region that must not allocate. The kept
// address is not valid after a cudaDeviceReset of that device.
#include <atomic>
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
// device address of g_scratch, per device; threads that race on the first
// call store the same value
static std::atomic<uint8_t*> g_addr[kMaxDevices];

static uint8_t* scratch_address(int* rc) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *rc = set_error_message(MOE_ERR_CUDA, "moe_matmul_q_dev_noalloc: no usable current device");
    return nullptr;
  }
  uint8_t* a = g_addr[dev].load(std::memory_order_acquire);
  if (!a) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p) {
      char msg[256];
      snprintf(msg, sizeof(msg), "moe_matmul_q_dev_noalloc: cudaGetSymbolAddress failed: %s",
               cudaGetErrorString(e));
      *rc = set_error_message(MOE_ERR_CUDA, msg);
      return nullptr;
    }
    a = static_cast<uint8_t*>(p);
    g_addr[dev].store(a, std::memory_order_release);
  }
  return a;
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
  const bool fast = K > 0 && ((uintptr_t)B_q % 16 == 0) && fast_geometry_ok(dtype, K);
  if (fast && (M > na::kMaxRows || (size_t)2 * M * K > na::kMaxPlaneBytes)) {
    snprintf(msg, sizeof(msg),
             "moe_matmul_q_dev_noalloc: M=%d K=%d exceeds the fixed scratch (M <= %d and M*K <= %zu)",
             M, K, na::kMaxRows, na::kMaxPlaneBytes / 2);
    return set_error_message(MOE_ERR_INVALID, msg);
  }
  if ((long)M * N == 0) return MOE_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 0) {
    // no products: C = 0, as moe_matmul_q8_dev / _q4_dev (B_s is not read)
    launch_zero_fill(C, (size_t)M * N, st);
    const cudaError_t e0 = cudaGetLastError();
    if (e0 != cudaSuccess) {
      snprintf(msg, sizeof(msg), "moe_matmul_q_dev_noalloc: %s", cudaGetErrorString(e0));
      return set_error_message(MOE_ERR_CUDA, msg);
    }
    return MOE_OK;
  }
  int rc = MOE_OK;
  uint8_t* base = na::scratch_address(&rc);
  if (!base) return rc;
  int* flag = reinterpret_cast<int*>(base);
  int* asum = reinterpret_cast<int*>(base + na::kHeaderBytes);
  uint8_t* act = base + na::kHeaderBytes + na::kSumBytes;
  cudaError_t e = cudaSuccess;
  {
    if (fast) {
      // truncated activation planes in the static array, then the warp GEMV,
      // which computes C exactly instead if any activation was out of range
      const int mark = next_range_mark();   // the error word needs no clearing
      launch_quantize_act(A, M, K, dtype, act, 2 * K, asum, flag, st, 0, nullptr, mark);
      const uint8_t* wq = static_cast<const uint8_t*>(B_q);
      launch_gemv(dtype, &wq, &B_s, 1, false, N, K, act, 2 * K, asum, M, C, st, A, flag, mark);
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
