// tmap.cuh — host helpers shared by the tensor-core kernels: TMA tensor maps
// (built through the driver entry point, no libcuda link), the SM count and
// the residency / cache-policy switches.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>
#include <mutex>
#include <unordered_map>
#include "kernels.cuh"

// Q4 decode keeps the expanded weights in tensor memory (moe_mma.cu)
#ifndef MOE_Q4_TMEM
#define MOE_Q4_TMEM 1
#endif

namespace moe {
namespace mm {

struct __align__(64) TMap { CUtensorMap m; };

static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// uint8 tensor map, 128-byte inner box with 128-byte swizzle. The encoding
// is a pure function of its arguments, and the same few maps (resident
// weight slabs, workspace planes) recur on every call, so encodings are
// memoised: a host call then costs no driver encode calls.
struct MapKey {
  const void* base; int rank, swizzle;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  bool operator==(const MapKey& o) const { return memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
    size_t h = 1469598103934665603ull;                 // FNV-1a over the key bytes
    for (size_t i = 0; i < sizeof(MapKey); ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
  }
};
static bool map_u8(TMap& t, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                   const cuuint32_t* box, bool swizzle = true) {
  static std::mutex mu;
  static std::unordered_map<MapKey, TMap, MapKeyHash> cache;
  MapKey k;
  memset(&k, 0, sizeof(k));
  k.base = base; k.rank = rank; k.swizzle = swizzle ? 1 : 0;
  for (int i = 0; i < rank; ++i) { k.dims[i] = dims[i]; k.box[i] = box[i]; }
  for (int i = 0; i + 1 < rank; ++i) k.strides[i] = strides[i];
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(k);
  if (it != cache.end()) { t = it->second; return true; }
  auto fn = encoder();
  if (!fn) return false;
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(&t.m, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(k, t);
  return true;
}

// weights of one projection over all local experts: (row bytes, rows, expert),
// 128-byte boxes with 128-byte swizzle. Q8: the MMA operand layout itself;
// Q4: 256 packed nibbles per row (two k-chunks), expanded in shared memory.
static bool map_weights(TMap& t, const LayerDev& L, size_t off, int kelems, int rows) {
  const bool q4 = L.dtype == 3;
  const int rb = q4 ? kelems / 2 : kelems;
  const cuuint64_t dims[3] = {(cuuint64_t)rb, (cuuint64_t)rows, (cuuint64_t)(L.e_end - L.e_begin)};
  const cuuint64_t strides[2] = {(cuuint64_t)rb, (cuuint64_t)L.expert_stride};
  const cuuint32_t box[3] = {128u, 128, 1};
  return map_u8(t, L.slab + off, 3, dims, strides, box, true);
}

// activation rows: (K bytes, J rows, row pitch); J >= the box height
static bool map_rows(TMap& t, const uint8_t* base, int kbytes, int J, int nt, int pitch = 0) {
  const cuuint64_t dims[2] = {(cuuint64_t)kbytes, (cuuint64_t)J};
  const cuuint64_t strides[1] = {(cuuint64_t)(pitch ? pitch : kbytes)};
  const cuuint32_t box[2] = {128, (cuuint32_t)nt};
  return map_u8(t, base, 2, dims, strides, box);
}

// Resident CTAs per SM. Two independent producer/MMA/epilogue pipelines per
// SM measured faster than one with twice the stages (T=16 decode: gate/up 58
// -> 51 us, down 39 -> 32 us); three leave too few stages. MOE_MMA_CTAS
// overrides, for tuning runs.
static int ctas_per_sm() {
  static int c = 0;
  if (!c) {
    const char* e = getenv("MOE_MMA_CTAS");
    c = e ? atoi(e) : 2;
    if (c < 1 || c > 3) c = 2;
  }
  return c;
}

static int sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Q4 stages carry the packed staging tiles too, so Q4 runs one CTA per SM
// with the whole shared-memory budget.
// Q4 decode tiles (expanded weights in TMEM, no shared-memory ring) run two
// CTAs per SM like Q8: two MMA issuers per SM.
static int ctas_for(int dt, int nt = 0) {
  const bool q4_two = MOE_Q4_TMEM && nt > 0 && nt <= 32;
  return dt == 4 ? (q4_two ? 2 : 1) : ctas_per_sm();
}
static int grid_ctas(int dt, int nt = 0) { return sms() * ctas_for(dt, nt); }
// weights read once per call are loaded evict-first (MOE_NO_EVICT_FIRST=1
// turns it off, for measurements)
static bool evict_first_on() {
  static int v = -1;
  if (v < 0) v = getenv("MOE_NO_EVICT_FIRST") ? 0 : 1;
  return v == 1;
}

}  // namespace mm
}  // namespace moe
