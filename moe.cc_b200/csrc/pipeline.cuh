// pipeline.cuh — mbarrier + 1-D bulk async copy (TMA engine) primitives for
// sm_100a, with bounded waits: a wait that exceeds its time limit (read from
// the GPU's %globaltimer, in nanoseconds) returns false instead of spinning
// forever, so a kernel can flag an error and leave cleanly.
#pragma once
#include <stdint.h>

namespace moe {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Nanoseconds of the GPU's global timer.
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Time limit of one wait on a local event (a copy landing, a pipeline stage
// freed, another CTA of the same kernel finishing a unit): those take
// microseconds, so 200 ms only ever expires when something is broken.
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;

// Wait for phase `parity` to complete; false once `limit_ns` has passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// global -> shared bulk copy (no multicast), completion counted on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- cross-GPU flags (expert-parallel exchange over peer memory) ----------
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// One thread: wait until flags[0..world) all reached seq. Bounded: a rank
// that never arrives makes this return false once limit_ns has passed since
// the wait began (one limit for the whole wait, not per flag), instead of
// hanging the GPU.
__device__ __forceinline__ bool wait_flags_sys(const unsigned long long* flags, int world,
                                               unsigned long long seq, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (int src = 0; src < world; ++src) {
    uint32_t i = 0;
    while (ld_acquire_sys(flags + src) < seq)
      if ((++i & 63) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

}  // namespace moe
