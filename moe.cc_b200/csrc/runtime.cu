// runtime.cu — host side of libmoe_cuda: the extern "C" boundary declared in
// include/moe_cuda.h, device residency of the expert weights, the per-call
// workspace and the orchestration of the fused MoE block.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <map>
#include <tuple>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/moe_cuda.h"
#include "common.cuh"
#include "kernels.cuh"

namespace moe {

struct Alias { const void* dev; size_t bytes; };

struct State {
  bool init = false;
  int device = 0, ep_world = 1, ep_rank = 0, sm_count = 0;
  std::map<int, LayerDev> layers;
  std::unordered_map<const void*, Alias> alias;  // host q/s pointer -> device copy
  Workspace ws;
  int* d_err = nullptr;                          // kernel-flagged errors
  int* h_err = nullptr;                          // pinned, mapped host copy of d_err
  int* h_err_dev = nullptr;                      // h_err's device address
  std::string last_error;
  std::recursive_mutex mu;
};

static State g;

static int set_err(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g.last_error = buf;
  return code;
}

// Error reporting for entry points defined in other .cu files of the library.
int set_error_message(int code, const char* msg) { return set_err(code, "%s", msg); }

#define CU(call)                                                                         \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return set_err(MOE_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                     __FILE__, __LINE__);                                                \
  } while (0)

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

#ifdef MOE_TIMELINE
void tl_io_router(unsigned long long*, int);
void tl_io_moe_mma(unsigned long long*, int);
void tl_io_ep(unsigned long long*, int);
void tl_io_moe_fused(unsigned long long*, int);
void fz_trace_read(unsigned long long*);
void q4_trace_read(long long*);
#endif

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) { const char* e = getenv("MOE_PDL"); v = e ? atoi(e) != 0 : 1; }
  return v == 1;
}

static int ensure_init() {
  if (!g.init) return set_err(MOE_ERR_NOT_INIT, "moe_cuda_init() has not been called");
  return MOE_OK;
}

// ---- graph replay of host-pointer moe_ffn calls (MOE_E2E_GRAPH=1) ----------
// A host-pointer call is: two host-to-device copies, the kernels, two or
// three device-to-host copies and the error-word readback. With the switch
// on, each (layer, T, flags, outputs) key is captured once into a CUDA graph
// (kernels as a child graph between explicit memcpy nodes) and replayed with
// one launch; only the memcpy nodes' host pointers change between calls.
// The graphs hold workspace and layer pointers, so every event that moves
// them (workspace growth, upload, free, shutdown) drops the cache.
struct HostGraph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaGraphNode_t in_xn = nullptr, in_xo = nullptr, out_xo = nullptr, out_idx = nullptr, out_p = nullptr;
  int eager_calls = 0;     // calls made eagerly before the capture (sets kernel attributes)
  bool failed = false;     // capture or instantiation refused: this key stays eager
};
static std::map<std::tuple<int, int, int, bool, bool>, HostGraph> g_host_graphs;
static cudaStream_t g_host_stream = nullptr;

static void host_graphs_reset() {
  for (auto& kv : g_host_graphs) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
  }
  g_host_graphs.clear();
}

static bool e2e_graph_on() {
  static int v = -1;
  if (v < 0) { const char* e = getenv("MOE_E2E_GRAPH"); v = e && atoi(e) != 0; }
  return v == 1;
}

// Grow the workspace to hold T tokens for a layer of shape (E, D, F, K).
static int ensure_workspace(int T, int E, int D, int F, int K) {
  Workspace& w = g.ws;
  if (T <= w.cap_T && E <= w.cap_E && D <= w.cap_D && F <= w.cap_F && K <= w.cap_K) return MOE_OK;
  host_graphs_reset();
  int nT = T > w.cap_T ? (T > 2 * w.cap_T ? T : 2 * w.cap_T) : w.cap_T;
  if (nT < 32) nT = 32;  // >= the widest decode tile: token rows are read as a tile
  const int nE = E > w.cap_E ? E : w.cap_E, nD = D > w.cap_D ? D : w.cap_D;
  const int nF = F > w.cap_F ? F : w.cap_F, nK = K > w.cap_K ? K : w.cap_K;
  CU(cudaDeviceSynchronize());
  void* ptrs[] = {w.logits, w.topk_idx, w.topk_p, w.route, w.xact, w.xsum, w.hact, w.hsum,
                  w.y, w.xn, w.xo, w.xs0, w.xs1, w.hs0, w.hs1, w.slot_pos, w.route_counter,
                  w.fused_ctr, w.xbad, w.xsum_s};
  for (void* p : ptrs) if (p) cudaFree(p);
  w = Workspace{};
  const size_t TK = (size_t)nT * nK;
  const size_t max_tiles = (size_t)route_max_tiles((int)TK, nE, 16);
#define ALLOC(field, bytes)                                                    \
  do {                                                                         \
    if (cudaMalloc((void**)&w.field, (bytes)) != cudaSuccess) {                \
      w = Workspace{};                                                         \
      return set_err(MOE_ERR_NOMEM, "workspace allocation of %zu bytes failed", \
                     (size_t)(bytes));                                         \
    }                                                                          \
  } while (0)
  ALLOC(logits, sizeof(float) * (size_t)nT * nE);
  ALLOC(topk_idx, sizeof(int) * TK);
  ALLOC(topk_p, sizeof(float) * TK);
  ALLOC(route, sizeof(int) * (2 + 2 * (size_t)nE + TK + 1 + 3 * max_tiles));
  ALLOC(xact, (size_t)2 * nD * nT);
  ALLOC(xsum, sizeof(int) * (size_t)nT);
  ALLOC(xsum_s, sizeof(int) * TK);
  ALLOC(hact, (size_t)2 * nF * TK);
  ALLOC(hsum, sizeof(int) * TK);
  ALLOC(y, sizeof(float) * TK * nD);
  ALLOC(xs0, TK * nD);
  ALLOC(xs1, TK * nD);
  ALLOC(hs0, TK * nF);
  ALLOC(hs1, TK * nF);
  ALLOC(slot_pos, sizeof(int) * TK);
  ALLOC(route_counter, sizeof(int));
  ALLOC(xn, sizeof(float) * (size_t)nT * nD);
  ALLOC(xo, sizeof(float) * (size_t)nT * nD);
  ALLOC(fused_ctr, sizeof(int) * (3 + 2 * kFusedMaxTiles));
  ALLOC(xbad, sizeof(int) * (2 + (size_t)nT));
#undef ALLOC
  CU(cudaMemset(w.xbad, 0, sizeof(int) * (2 + (size_t)nT)));
  CU(cudaMemset(w.fused_ctr, 0, sizeof(int) * (3 + 2 * kFusedMaxTiles)));
  CU(cudaMemset(w.route_counter, 0, sizeof(int)));
  w.cap_T = nT; w.cap_E = nE; w.cap_D = nD; w.cap_F = nF; w.cap_K = nK;
  return MOE_OK;
}

// Read (and clear) the kernel error flag. Synchronises the device.
static int error_status(int h) {
  if (h) {
    // a timeout is reported first: it means some kernel's results are missing
    if (h & kErrTimeout)
      return set_err(MOE_ERR_CUDA,
                     "a kernel gave up waiting (bounded wait on a copy, or on another rank's flag)");
    if (h & kErrRange)
      return set_err(MOE_ERR_RANGE,
                     "an activation was NaN/inf or outside the integer range of the "
                     "quantised kernels (Q8: |x| < 258, Q4: trunc(7x) in [-128,127])");
  }
  return MOE_OK;
}

static int consume_device_error() {
  int h = 0;
  CU(cudaDeviceSynchronize());
  CU(cudaMemcpy(&h, g.d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h) CU(cudaMemset(g.d_err, 0, sizeof(int)));
  return error_status(h);
}

// The error flag as of the work queued on `st`: an async copy into pinned
// host memory and one stream synchronisation (no device-wide sync), for the
// synchronous host-pointer entry points.
static int consume_stream_error(cudaStream_t st, bool published = false) {
  if (!published) CU(cudaMemcpyAsync(g.h_err, g.d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  CU(cudaStreamSynchronize(st));
  const int h = *g.h_err;
  if (h) {
    *g.h_err = 0;
    CU(cudaMemsetAsync(g.d_err, 0, sizeof(int), st));
    CU(cudaStreamSynchronize(st));
  }
  return error_status(h);
}

// The device address of [p, p + bytes) when the whole range lies in ONE
// page-locked host allocation mapped into the device's address space
// (cudaHostAlloc, cudaMallocHost, cudaHostRegister); null otherwise
// (pageable memory, device memory, a range that spans allocations). Both
// ends are looked up and must carry the same allocation id, so a kernel
// given the address touches no unmapped page.
static void* mapped_host_range(const void* p, size_t bytes) {
  static PFN_cuPointerGetAttribute_v4000 get = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get = reinterpret_cast<PFN_cuPointerGetAttribute_v4000>(fn);
  }
  if (!get || !p || bytes == 0) return nullptr;
  const uintptr_t first = (uintptr_t)p, last = first + bytes - 1;
  cudaPointerAttributes a{}, b{};
  if (cudaPointerGetAttributes(&a, (const void*)first) != cudaSuccess ||
      cudaPointerGetAttributes(&b, (const void*)last) != cudaSuccess) {
    cudaGetLastError();          // pageable memory on older runtimes reports an error; clear it
    return nullptr;
  }
  if (a.type != cudaMemoryTypeHost || b.type != cudaMemoryTypeHost || !a.devicePointer || !b.devicePointer)
    return nullptr;
  unsigned long long ia = 0, ib = 0;
  if (get(&ia, CU_POINTER_ATTRIBUTE_BUFFER_ID, (CUdeviceptr)first) != CUDA_SUCCESS ||
      get(&ib, CU_POINTER_ATTRIBUTE_BUFFER_ID, (CUdeviceptr)last) != CUDA_SUCCESS || ia != ib)
    return nullptr;
  if ((uintptr_t)b.devicePointer - (uintptr_t)a.devicePointer != bytes - 1) return nullptr;
  return a.devicePointer;
}

}  // namespace moe

using namespace moe;

// ---------------------------------------------------------------------------
// scratch for the matmul_* entry points (grown on demand, never shrunk)
// ---------------------------------------------------------------------------
namespace moe {
static void ep_shutdown_hook();   // releases the expert-parallel buffers (defined below)
struct Buf { void* p = nullptr; size_t cap = 0; };
static Buf s_A, s_C, s_W, s_S, s_act, s_asum, s_hf, s_flag;

int next_range_mark() {
  static std::atomic<unsigned> n{0};
  unsigned v;
  while ((v = ++n) == 0u) {}            // never 0 (0 means "no mark")
  return (int)v;
}

static int grow(Buf& b, size_t bytes) {
  if (bytes <= b.cap) return MOE_OK;
  if (b.p) { CU(cudaDeviceSynchronize()); cudaFree(b.p); b.p = nullptr; b.cap = 0; }
  size_t n = align_up(bytes, 1 << 20);
  if (cudaMalloc(&b.p, n) != cudaSuccess)
    return set_err(MOE_ERR_NOMEM, "scratch allocation of %zu bytes failed", n);
  b.cap = n;
  return MOE_OK;
}

static const void* lookup_alias(const void* host) {
  auto it = g.alias.find(host);
  return it == g.alias.end() ? nullptr : it->second.dev;
}

static int check_mnk(int M, int N, int K) {
  if (M < 0 || N < 0 || K < 0) return set_err(MOE_ERR_INVALID, "negative M/N/K (%d,%d,%d)", M, N, K);
  return MOE_OK;
}

// Q8/Q4 matmul on device pointers: activation truncation + the fast warp GEMV,
// which computes exactly from the fp32 activations instead when the
// truncation marked one outside the 16-bit / 8-bit range, so the result is
// the reference's for any activation magnitude.
static int matmul_q_dev(int dtype, const float* A, const void* Bq, const float* Bs, float* C,
                        int M, int N, int K, cudaStream_t st) {
  int rc = check_mnk(M, N, K);
  if (rc) return rc;
  if (dtype == MOE_DTYPE_Q4 && (K & 1))
    return set_err(MOE_ERR_UNSUPPORTED,
                   "Q4 with odd K=%d: the reference reads one byte past the packed row "
                   "(kernels.c:108,116); not reproduced", K);
  if ((long)M * N == 0) return MOE_OK;
  if (K == 0) { launch_zero_fill(C, (size_t)M * N, st); return MOE_OK; }
  const bool aligned = ((uintptr_t)Bq % 16 == 0);
  if (aligned && fast_geometry_ok(dtype, K)) {
    if ((rc = grow(s_act, (size_t)2 * K * M))) return rc;
    if ((rc = grow(s_asum, sizeof(int) * (size_t)M))) return rc;
    if ((rc = grow(s_flag, sizeof(int)))) return rc;
    int* flag = (int*)s_flag.p;
    const int mark = next_range_mark();
    launch_quantize_act(A, M, K, dtype, (uint8_t*)s_act.p, 2 * K, (int*)s_asum.p, flag, st, 0, nullptr, mark);
    const uint8_t* wq = (const uint8_t*)Bq;
    launch_gemv(dtype, &wq, &Bs, 1, false, N, K, (const uint8_t*)s_act.p, 2 * K,
                  (const int*)s_asum.p, M, C, st, A, flag, mark);
  } else {
    launch_gemv_generic(dtype, A, (const uint8_t*)Bq, Bs, C, M, N, K, st);
  }
  CU(cudaGetLastError());
  return MOE_OK;
}

// Host-pointer synchronous matmul (the reference's calling convention).
static int matmul_q_host(int dtype, const float* A, const void* Bq, const float* Bs, float* C,
                         int M, int N, int K) {
  int rc = ensure_init();
  if (rc) return rc;
  if ((rc = check_mnk(M, N, K))) return rc;
  if ((long)M * N == 0) return MOE_OK;
  const size_t wbytes = (size_t)N * (dtype == MOE_DTYPE_Q8 ? K : K / 2);
  const void* dq = lookup_alias(Bq);
  const float* ds = (const float*)lookup_alias(Bs);
  if (!dq || !ds) {
    if ((rc = grow(s_W, wbytes + 16)) || (rc = grow(s_S, sizeof(float) * (size_t)N))) return rc;
    CU(cudaMemcpy(s_W.p, Bq, wbytes, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(s_S.p, Bs, sizeof(float) * N, cudaMemcpyHostToDevice));
    dq = s_W.p; ds = (const float*)s_S.p;
  }
  if ((rc = grow(s_A, sizeof(float) * (size_t)M * K + 16)) ||
      (rc = grow(s_C, sizeof(float) * (size_t)M * N)))
    return rc;
  CU(cudaMemcpy(s_A.p, A, sizeof(float) * (size_t)M * K, cudaMemcpyHostToDevice));
  if ((rc = matmul_q_dev(dtype, (const float*)s_A.p, dq, ds, (float*)s_C.p, M, N, K, 0))) return rc;
  if ((rc = consume_stream_error(0))) return rc;
  CU(cudaMemcpy(C, s_C.p, sizeof(float) * (size_t)M * N, cudaMemcpyDeviceToHost));
  return MOE_OK;
}

static void die_on(int rc, const char* who) {
  if (rc == MOE_OK) return;
  fprintf(stderr, "libmoe_cuda: %s failed (%d): %s\n", who, rc, g.last_error.c_str());
  abort();
}
}  // namespace moe

extern "C" {

int moe_cuda_init(int device, int ep_world, int ep_rank, const void* nccl_uid) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  if (nccl_uid) return set_err(MOE_ERR_UNSUPPORTED, "nccl_uid must be NULL");
  if (ep_world < 1 || ep_rank < 0 || ep_rank >= ep_world)
    return set_err(MOE_ERR_INVALID, "bad expert-parallel group (world %d rank %d)", ep_world, ep_rank);
  if (g.init) {
    if (device == g.device && ep_world == g.ep_world && ep_rank == g.ep_rank) return MOE_OK;
    return set_err(MOE_ERR_INVALID, "already initialised on device %d (world %d rank %d)",
                   g.device, g.ep_world, g.ep_rank);
  }
  CU(cudaSetDevice(device));
  CU(cudaDeviceGetAttribute(&g.sm_count, cudaDevAttrMultiProcessorCount, device));
  CU(cudaMalloc((void**)&g.d_err, sizeof(int)));
  CU(cudaMemset(g.d_err, 0, sizeof(int)));
  CU(cudaHostAlloc((void**)&g.h_err, sizeof(int), cudaHostAllocMapped));
  CU(cudaHostGetDevicePointer((void**)&g.h_err_dev, g.h_err, 0));
  *g.h_err = 0;
  g.device = device; g.ep_world = ep_world; g.ep_rank = ep_rank;
  g.init = true;
  return MOE_OK;
}

int moe_cuda_shutdown(void) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  if (!g.init) return MOE_OK;
  cudaDeviceSynchronize();
  host_graphs_reset();
  if (g_host_stream) { cudaStreamDestroy(g_host_stream); g_host_stream = nullptr; }
  ep_shutdown_hook();
  for (auto& kv : g.layers) {
    cudaFree(kv.second.slab); cudaFree(kv.second.router_w);
    if (kv.second.router_b) cudaFree(kv.second.router_b);
  }
  g.layers.clear();
  g.alias.clear();
  Workspace& w = g.ws;
  void* ptrs[] = {w.logits, w.topk_idx, w.topk_p, w.route, w.xact, w.xsum, w.hact, w.hsum,
                  w.y, w.xn, w.xo, w.xs0, w.xs1, w.hs0, w.hs1, w.slot_pos, w.route_counter,
                  w.fused_ctr, w.xbad, w.xsum_s};
  for (void* p : ptrs) if (p) cudaFree(p);
  w = Workspace{};
  Buf* bufs[] = {&s_A, &s_C, &s_W, &s_S, &s_act, &s_asum, &s_hf, &s_flag};
  for (Buf* b : bufs) { if (b->p) cudaFree(b->p); *b = Buf{}; }
  cudaFree(g.d_err); g.d_err = nullptr;
  if (g.h_err) cudaFreeHost(g.h_err);
  g.h_err = nullptr;
  g.init = false;
  return MOE_OK;
}

const char* moe_cuda_last_error(void) { return g.last_error.c_str(); }

int moe_cuda_check_status(void) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  int rc = ensure_init();
  if (rc) return rc;
  CU(cudaGetLastError());
  return consume_device_error();
}

void matmul_f32_q8(const float* A, const int8_t* B_q, const float* B_s, float* C, int M, int N, int K) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  die_on(matmul_q_host(MOE_DTYPE_Q8, A, B_q, B_s, C, M, N, K), "matmul_f32_q8");
}

void matmul_f32_q4(const float* A, const uint8_t* B_q, const float* B_s, float* C, int M, int N, int K) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  die_on(matmul_q_host(MOE_DTYPE_Q4, A, B_q, B_s, C, M, N, K), "matmul_f32_q4");
}

static int matmul_f32_host(const float* A, const float* W, float* C, int M, int N, int K) {
  int rc = ensure_init();
  if (rc || (rc = check_mnk(M, N, K))) return rc;
  if ((long)M * N == 0) return MOE_OK;
  const float* dW = (const float*)lookup_alias(W);
  if (!dW) {
    if ((rc = grow(s_W, sizeof(float) * (size_t)N * K + 16))) return rc;
    CU(cudaMemcpy(s_W.p, W, sizeof(float) * (size_t)N * K, cudaMemcpyHostToDevice));
    dW = (const float*)s_W.p;
  }
  if ((rc = grow(s_A, sizeof(float) * (size_t)M * K + 16)) ||
      (rc = grow(s_C, sizeof(float) * (size_t)M * N)))
    return rc;
  CU(cudaMemcpy(s_A.p, A, sizeof(float) * (size_t)M * K, cudaMemcpyHostToDevice));
  launch_f32_seq_matmul((const float*)s_A.p, dW, nullptr, (float*)s_C.p, M, N, K, 0);
  CU(cudaGetLastError());
  CU(cudaMemcpy(C, s_C.p, sizeof(float) * (size_t)M * N, cudaMemcpyDeviceToHost));
  return MOE_OK;
}

void matmul_adaptive(const float* A, const float* W_fp32, const void* W_q_ptr, float* C, int M,
                     int N, int K) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const QuantizedWeight* w = (const QuantizedWeight*)W_q_ptr;
  int rc;
  if (!w) rc = matmul_f32_host(A, W_fp32, C, M, N, K);
  else if (w->dtype == MOE_DTYPE_Q8 || w->dtype == MOE_DTYPE_Q4)
    rc = matmul_q_host(w->dtype, A, w->q, w->s, C, M, N, K);
  else {
    // unsupported dtype: zero output, as kernels.c:172-180
    if (M > 0 && N > 0) memset(C, 0, sizeof(float) * (size_t)M * N);
    rc = MOE_OK;
  }
  die_on(rc, "matmul_adaptive");
}

int moe_matmul_q8_dev(const float* A, const int8_t* B_q, const float* B_s, float* C, int M, int N,
                      int K, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  int rc = ensure_init();
  return rc ? rc : matmul_q_dev(MOE_DTYPE_Q8, A, B_q, B_s, C, M, N, K, (cudaStream_t)stream);
}

int moe_matmul_q4_dev(const float* A, const uint8_t* B_q, const float* B_s, float* C, int M, int N,
                      int K, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  int rc = ensure_init();
  return rc ? rc : matmul_q_dev(MOE_DTYPE_Q4, A, B_q, B_s, C, M, N, K, (cudaStream_t)stream);
}

int moe_matmul_f32_dev(const float* A, const float* W, float* C, int M, int N, int K, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  int rc = ensure_init();
  if (rc || (rc = check_mnk(M, N, K))) return rc;
  launch_f32_seq_matmul(A, W, nullptr, C, M, N, K, (cudaStream_t)stream);
  CU(cudaGetLastError());
  return MOE_OK;
}

int moe_matmul_batched_dev(const float* A, const void* const* W_q, const float* const* W_s, float* C,
                           int n_mat, int N, int K, int dtype, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  int rc = ensure_init();
  if (rc) return rc;
  if (dtype != MOE_DTYPE_Q8 && dtype != MOE_DTYPE_Q4) return set_err(MOE_ERR_INVALID, "dtype %d", dtype);
  if (n_mat <= 0 || N <= 0 || K <= 0) return set_err(MOE_ERR_INVALID, "empty batched matmul");
  if (!fast_geometry_ok(dtype, K))
    return set_err(MOE_ERR_UNSUPPORTED, "batched matmul needs K with 16-byte rows (K=%d)", K);
  cudaStream_t st = (cudaStream_t)stream;
  if ((rc = grow(s_act, (size_t)2 * K)) || (rc = grow(s_asum, sizeof(int))) || (rc = grow(s_flag, sizeof(int))))
    return rc;
  int* flag = (int*)s_flag.p;
  const int mark = next_range_mark();
  launch_quantize_act(A, 1, K, dtype, (uint8_t*)s_act.p, 2 * K, (int*)s_asum.p, flag, st, 0, nullptr, mark);
  // (an activation out of the fast range makes the GEMV compute exactly)
  launch_gemv(dtype, (const uint8_t* const*)W_q, W_s, n_mat, true, N, K, (const uint8_t*)s_act.p,
                2 * K, (const int*)s_asum.p, 1, C, st, A, flag, mark);
  CU(cudaGetLastError());
  return MOE_OK;
}

int moe_quantize_rowwise_q8_dev(const float* W, int rows, int cols, int8_t* q, float* s, void* stream) {
  if (rows < 0 || cols <= 0) return set_err(MOE_ERR_INVALID, "bad shape %dx%d", rows, cols);
  launch_quantize_rowwise(MOE_DTYPE_Q8, W, rows, cols, q, s, (cudaStream_t)stream);
  CU(cudaGetLastError());
  return MOE_OK;
}

int moe_quantize_rowwise_q4_dev(const float* W, int rows, int cols, uint8_t* q, float* s, void* stream) {
  if (rows < 0 || cols <= 0 || (cols & 1))
    return set_err(MOE_ERR_INVALID, "Q4 needs an even column count (%dx%d)", rows, cols);
  launch_quantize_rowwise(MOE_DTYPE_Q4, W, rows, cols, q, s, (cudaStream_t)stream);
  CU(cudaGetLastError());
  return MOE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// weight residency + fused MoE block
// ---------------------------------------------------------------------------
namespace moe {

static int validate_layer(const QuantizedWeight* Wg, const QuantizedWeight* Wu,
                          const QuantizedWeight* Wd, int E, int* D, int* F, int* dtype) {
  if (E <= 0 || !Wg || !Wu || !Wd) return set_err(MOE_ERR_INVALID, "empty layer (E=%d)", E);
  // the router keeps the top 8 (test_model_trace.c:475-478, top_k fixed at 8
  // by model.h:160)
  if (E < 8) return set_err(MOE_ERR_UNSUPPORTED, "top-8 routing needs at least 8 experts (E=%d)", E);
  *dtype = Wg[0].dtype; *F = Wg[0].rows; *D = Wg[0].cols;
  if (*dtype != MOE_DTYPE_Q8 && *dtype != MOE_DTYPE_Q4)
    return set_err(MOE_ERR_UNSUPPORTED, "expert dtype %d (only Q8=2 / Q4=3)", *dtype);
  for (int e = 0; e < E; ++e) {
    const QuantizedWeight* w[3] = {&Wg[e], &Wu[e], &Wd[e]};
    for (int i = 0; i < 3; ++i) {
      const int rows = i < 2 ? *F : *D, cols = i < 2 ? *D : *F;
      if (w[i]->dtype != *dtype || w[i]->rows != rows || w[i]->cols != cols || !w[i]->q || !w[i]->s)
        return set_err(MOE_ERR_INVALID, "expert %d projection %d: shape/dtype mismatch", e, i);
    }
  }
  if (!fast_geometry_ok(*dtype, *D) || !fast_geometry_ok(*dtype, *F))
    return set_err(MOE_ERR_UNSUPPORTED,
                   "moe_ffn needs D and F whose packed rows are multiples of 16 bytes "
                   "(D=%d F=%d dtype %d)", *D, *F, *dtype);
  return MOE_OK;
}

// Pinned staging for streamed uploads: two expert-slab images, filled on the
// host while the other one's copy runs; released after the stream drains.
struct PinnedRing {
  uint8_t* buf[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  cudaStream_t st = nullptr;
  ~PinnedRing() {
    if (st) cudaStreamSynchronize(st);
    for (int i = 0; i < 2; ++i) {
      if (buf[i]) cudaFreeHost(buf[i]);
      if (ev[i]) cudaEventDestroy(ev[i]);
    }
    if (st) cudaStreamDestroy(st);
  }
};

// register_alias: remember the host q/s pointers for the matmul_* drop-ins
// (not for staging memory the caller frees right after the upload).
// reader: when set, the experts' q/s pointers are placeholders and each local
// expert's slab image is produced by reader->fill into pinned memory instead,
// double-buffered against its host-to-device copy.
static int upload_layer(int layer, const QuantizedWeight* Wg, const QuantizedWeight* Wu,
                        const QuantizedWeight* Wd, const float* router_w, const float* router_b,
                        int E, cudaMemcpyKind kind, bool register_alias = true,
                        const ExpertReader* reader = nullptr) {
  int rc = ensure_init();
  if (rc) return rc;
  int D, F, dtype;
  if ((rc = validate_layer(Wg, Wu, Wd, E, &D, &F, &dtype))) return rc;
  if (!router_w) return set_err(MOE_ERR_INVALID, "router_w is NULL");
  host_graphs_reset();
  if (g.layers.count(layer)) moe_cuda_free_layer(layer);
  LayerDev L;
  L.E = E; L.D = D; L.F = F; L.dtype = dtype; L.topk = 8;
  L.e_begin = (int)((long)E * g.ep_rank / g.ep_world);
  L.e_end = (int)((long)E * (g.ep_rank + 1) / g.ep_world);
  L.gu_rb = dtype == MOE_DTYPE_Q8 ? D : D / 2;
  L.d_rb = dtype == MOE_DTYPE_Q8 ? F : F / 2;
  const size_t gub = (size_t)F * L.gu_rb, db = (size_t)D * L.d_rb;
  L.gq_off = 0;
  L.uq_off = align_up(gub, 128);
  L.dq_off = L.uq_off + align_up(gub, 128);
  L.gs_off = L.dq_off + align_up(db, 128);
  L.us_off = L.gs_off + align_up(sizeof(float) * F, 128);
  L.ds_off = L.us_off + align_up(sizeof(float) * F, 128);
  L.expert_stride = align_up(L.ds_off + sizeof(float) * D, 128);
  const int El = L.e_end - L.e_begin;
  L.bytes = L.expert_stride * (size_t)(El > 0 ? El : 0);
  if (El > 0 && cudaMalloc((void**)&L.slab, L.bytes) != cudaSuccess)
    return set_err(MOE_ERR_NOMEM, "layer %d: %zu bytes of expert slabs", layer, L.bytes);
  if (cudaMalloc((void**)&L.router_w, sizeof(float) * (size_t)E * D) != cudaSuccess) {
    cudaFree(L.slab);
    return set_err(MOE_ERR_NOMEM, "layer %d router", layer);
  }
  if (router_b && cudaMalloc((void**)&L.router_b, sizeof(float) * E) != cudaSuccess) {
    cudaFree(L.slab); cudaFree(L.router_w);
    return set_err(MOE_ERR_NOMEM, "layer %d router bias", layer);
  }
  g.layers[layer] = L;  // registered before the copies so free_layer cleans up on error
  CU(cudaMemcpy(L.router_w, router_w, sizeof(float) * (size_t)E * D, kind));
  if (router_b) CU(cudaMemcpy(L.router_b, router_b, sizeof(float) * E, kind));
  if (reader) {
    PinnedRing ring;
    CU(cudaStreamCreateWithFlags(&ring.st, cudaStreamNonBlocking));
    for (int i = 0; i < 2 && i < El; ++i) {
      CU(cudaHostAlloc((void**)&ring.buf[i], L.expert_stride, cudaHostAllocDefault));
      memset(ring.buf[i], 0, L.expert_stride);     // alignment padding stays zero
      CU(cudaEventCreateWithFlags(&ring.ev[i], cudaEventDisableTiming));
    }
    for (int e = L.e_begin; e < L.e_end; ++e) {
      const int i = (e - L.e_begin) & 1;
      if (e - L.e_begin >= 2) CU(cudaEventSynchronize(ring.ev[i]));
      if (!reader->fill(reader->ctx, e, L, ring.buf[i])) {
        cudaStreamSynchronize(ring.st);
        moe_cuda_free_layer(layer);
        return MOE_ERR_INVALID;                      // the reader set the message
      }
      CU(cudaMemcpyAsync(L.slab + (size_t)(e - L.e_begin) * L.expert_stride, ring.buf[i], L.expert_stride,
                         cudaMemcpyHostToDevice, ring.st));
      CU(cudaEventRecord(ring.ev[i], ring.st));
    }
    CU(cudaStreamSynchronize(ring.st));
    return MOE_OK;
  }
  for (int e = L.e_begin; e < L.e_end; ++e) {
    uint8_t* base = L.slab + (size_t)(e - L.e_begin) * L.expert_stride;
    struct Part { const void* src; size_t off, bytes; } parts[6] = {
        {Wg[e].q, L.gq_off, gub}, {Wu[e].q, L.uq_off, gub}, {Wd[e].q, L.dq_off, db},
        {Wg[e].s, L.gs_off, sizeof(float) * F}, {Wu[e].s, L.us_off, sizeof(float) * F},
        {Wd[e].s, L.ds_off, sizeof(float) * D}};
    for (const Part& p : parts) {
      CU(cudaMemcpy(base + p.off, p.src, p.bytes, kind));
      if (kind == cudaMemcpyHostToDevice && register_alias) g.alias[p.src] = Alias{base + p.off, p.bytes};
    }
  }
  if (kind == cudaMemcpyHostToDevice && register_alias)
    g.alias[router_w] = Alias{L.router_w, sizeof(float) * (size_t)E * D};
  return MOE_OK;
}

// Optional per-kernel timing of moe_ffn (bench.py uses it for the roofline):
// events recorded on the launching stream around each launch.
struct ProfRec { const char* name; cudaEvent_t a, b; };
static bool g_prof = false;
static std::vector<ProfRec> g_prof_pending;
static std::map<std::string, std::pair<double, long>> g_prof_acc;

template <class F>
static void timed(const char* name, cudaStream_t st, F&& launch) {
  if (!g_prof) { launch(); return; }
  ProfRec r{name, nullptr, nullptr};
  cudaEventCreate(&r.a); cudaEventCreate(&r.b);
  cudaEventRecord(r.a, st);
  launch();
  cudaEventRecord(r.b, st);
  g_prof_pending.push_back(r);
}

static void prof_drain() {
  for (ProfRec& r : g_prof_pending) {
    float ms = 0.f;
    cudaEventSynchronize(r.b);
    cudaEventElapsedTime(&ms, r.a, r.b);
    auto& acc = g_prof_acc[r.name];
    acc.first += ms; acc.second += 1;
    cudaEventDestroy(r.a); cudaEventDestroy(r.b);
  }
  g_prof_pending.clear();
}

// Router + top-k + routing lists + token activation truncation.
// given: w.topk_idx / w.topk_p already hold the routing (MOE_FFN_GIVEN_TOPK):
// no router logits or top-k, only the activations and the routing lists.
// Routing of one call. res: an extra copy the decode routing kernel makes
// on the side; returns whether it was made (the other routing paths skip it).
static bool route_tokens(const LayerDev& L, const float* xn, int T, int nt, cudaStream_t st,
                         bool given = false, const RowCopy* res = nullptr) {
  if (!given && decode_route_supported(L, T, xn)) {
    timed("route", st, [&] {
      launch_decode_route(L, g.ws, xn, T, nt, g.ws.route_counter, g.d_err, st, nullptr, res);
    });
    return res != nullptr;
  }
  const Workspace& w = g.ws;
  timed("quantize_act", st, [&] {
    launch_quantize_act(xn, T, L.D, L.dtype, w.xact, 2 * L.D, w.xsum, g.d_err, st, nt > 0, w.xbad);
  });
  if (!given) {
    timed("router_logits", st, [&] {
      launch_f32_seq_matmul(xn, L.router_w, L.router_b, w.logits, T, L.E, L.D, st);
    });
    timed("topk_softmax", st, [&] {
      launch_topk_softmax(w.logits, T, L.E, L.topk, w.topk_idx, w.topk_p, st);
    });
  }
  timed("route_build", st, [&] {
    if (L.e_end - L.e_begin <= kRouteBuildMaxE)
      launch_route_build_multi(w.topk_idx, T, L.topk, L.e_begin, L.e_end - L.e_begin, w.route,
                               L.dtype == MOE_DTYPE_Q4 ? w.hsum : nullptr, nt,
                               nt > 0 ? w.slot_pos : nullptr, st);
    else
      launch_route_build(w.topk_idx, T, L.topk, L.e_begin, L.e_end, w.route, L.e_end - L.e_begin,
                         L.dtype == MOE_DTYPE_Q4 ? w.hsum : nullptr, nt, nt > 0 ? w.slot_pos : nullptr, st);
  });
  return false;
}

static int get_layer(int layer, const LayerDev** out) {
  int rc = ensure_init();
  if (rc) return rc;
  auto it = g.layers.find(layer);
  if (it == g.layers.end()) return set_err(MOE_ERR_NOT_INIT, "layer %d was not uploaded", layer);
  *out = &it->second;
  return MOE_OK;
}

static void run_gateup(const LayerDev& L, const Workspace& w, int T, cudaStream_t st) {
  launch_gateup(L, w, T, g.d_err, st);
}

static void run_down(const LayerDev& L, const Workspace& w, int T, float* y, cudaStream_t st) {
  launch_down(L, w, T, y, st);
}

// Tensor-core (tcgen05) expert GEMMs unless the caller forces the CUDA-core
// GEMVs (MOE_FFN_FORCE_GEMV, or MOE_FFN_PATH=gemv in the environment), or a
// call of at most kGemvMaxT tokens: one token's 8 experts make too few
// 128-row GEMM units to spread over the SMs, and the warp GEMVs, which spread
// every row over its own warp, measured faster there (T=1: 36.9 against
// 43.3 us per step).
constexpr int kGemvMaxT = 1;
static bool use_tensor_cores(const LayerDev& L, int flags, int T) {
  if (flags & MOE_FFN_FORCE_GEMV) return false;
  if (T <= kGemvMaxT && !(flags & MOE_FFN_FORCE_GEMM)) return false;
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("MOE_FFN_PATH");
    env = (e && strcmp(e, "gemv") == 0) ? 0 : 1;
  }
  if (!env && !(flags & MOE_FFN_FORCE_GEMM)) return false;
  return mma_supported(L);
}

// Captures the kernels of one host-pointer call into hg (between explicit
// memcpy nodes for the inputs, outputs and error word). False, with nothing
// kept, when the runtime refuses any step.
template <class Enqueue>
static bool build_host_graph(HostGraph& hg, cudaStream_t st, const float* x_norm2, float* x_inout, int* idx_out,
                             float* p_out, size_t xb, size_t kb, Enqueue& enqueue) {
  const Workspace& w = g.ws;
  cudaGraph_t kg = nullptr, gr = nullptr;
  if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return false;
  const int rc = enqueue(w.xn, w.xo, st);
  const cudaError_t ce = cudaStreamEndCapture(st, &kg);
  if (rc || ce != cudaSuccess || !kg) {
    if (kg) cudaGraphDestroy(kg);
    cudaGetLastError();
    return false;
  }
  const cudaMemcpyKind h2d = cudaMemcpyHostToDevice, d2h = cudaMemcpyDeviceToHost;
  cudaGraphNode_t child = nullptr, err = nullptr;
  bool ok = cudaGraphCreate(&gr, 0) == cudaSuccess;
  ok = ok && cudaGraphAddMemcpyNode1D(&hg.in_xn, gr, nullptr, 0, w.xn, x_norm2, xb, h2d) == cudaSuccess;
  ok = ok && cudaGraphAddMemcpyNode1D(&hg.in_xo, gr, nullptr, 0, w.xo, x_inout, xb, h2d) == cudaSuccess;
  cudaGraphNode_t ins[2] = {hg.in_xn, hg.in_xo};
  ok = ok && cudaGraphAddChildGraphNode(&child, gr, ins, 2, kg) == cudaSuccess;
  cudaGraphDestroy(kg);                          // the child node holds its own copy
  ok = ok && cudaGraphAddMemcpyNode1D(&hg.out_xo, gr, &child, 1, x_inout, w.xo, xb, d2h) == cudaSuccess;
  if (idx_out)
    ok = ok && cudaGraphAddMemcpyNode1D(&hg.out_idx, gr, &child, 1, idx_out, w.topk_idx, kb, d2h) == cudaSuccess;
  if (p_out)
    ok = ok && cudaGraphAddMemcpyNode1D(&hg.out_p, gr, &child, 1, p_out, w.topk_p, kb, d2h) == cudaSuccess;
  ok = ok && cudaGraphAddMemcpyNode1D(&err, gr, &child, 1, g.h_err, g.d_err, sizeof(int), d2h) == cudaSuccess;
  ok = ok && cudaGraphInstantiate(&hg.exec, gr, 0) == cudaSuccess;
  if (!ok) {
    if (hg.exec) cudaGraphExecDestroy(hg.exec);
    if (gr) cudaGraphDestroy(gr);
    hg = HostGraph{};
    cudaGetLastError();
    return false;
  }
  hg.graph = gr;
  return true;
}

// Host-pointer moe_ffn through a cached graph (MOE_E2E_GRAPH=1, stream NULL).
// The library's own blocking stream keeps the order the legacy stream gives
// the eager path. The first call of each key runs eagerly (it sets kernel
// attributes and encodes tensor maps outside any capture); any key whose
// capture, instantiation or node update the runtime refuses stays eager.
template <class Enqueue>
static int moe_ffn_host_graph(int layer, int T, int flags, const float* x_norm2, float* x_inout, int* idx_out,
                              float* p_out, size_t xb, size_t kb, Enqueue& enqueue) {
  const Workspace& w = g.ws;
  if (!g_host_stream) CU(cudaStreamCreate(&g_host_stream));
  cudaStream_t st = g_host_stream;
  HostGraph& hg = g_host_graphs[std::make_tuple(layer, T, flags, idx_out != nullptr, p_out != nullptr)];
  auto eager = [&]() -> int {
    CU(cudaMemcpyAsync(w.xn, x_norm2, xb, cudaMemcpyHostToDevice, st));
    CU(cudaMemcpyAsync(w.xo, x_inout, xb, cudaMemcpyHostToDevice, st));
    const int rc = enqueue(w.xn, w.xo, st);
    if (rc) return rc;
    if (idx_out) CU(cudaMemcpyAsync(idx_out, w.topk_idx, kb, cudaMemcpyDeviceToHost, st));
    if (p_out) CU(cudaMemcpyAsync(p_out, w.topk_p, kb, cudaMemcpyDeviceToHost, st));
    CU(cudaMemcpyAsync(x_inout, w.xo, xb, cudaMemcpyDeviceToHost, st));
    return consume_stream_error(st);
  };
  if (hg.failed || hg.eager_calls < 1) {
    hg.eager_calls++;
    return eager();
  }
  if (!hg.exec) {
    if (!build_host_graph(hg, st, x_norm2, x_inout, idx_out, p_out, xb, kb, enqueue)) {
      hg.failed = true;
      return eager();
    }
  } else {
    const cudaMemcpyKind h2d = cudaMemcpyHostToDevice, d2h = cudaMemcpyDeviceToHost;
    bool ok = cudaGraphExecMemcpyNodeSetParams1D(hg.exec, hg.in_xn, w.xn, x_norm2, xb, h2d) == cudaSuccess &&
              cudaGraphExecMemcpyNodeSetParams1D(hg.exec, hg.in_xo, w.xo, x_inout, xb, h2d) == cudaSuccess &&
              cudaGraphExecMemcpyNodeSetParams1D(hg.exec, hg.out_xo, x_inout, w.xo, xb, d2h) == cudaSuccess;
    if (ok && idx_out)
      ok = cudaGraphExecMemcpyNodeSetParams1D(hg.exec, hg.out_idx, idx_out, w.topk_idx, kb, d2h) == cudaSuccess;
    if (ok && p_out)
      ok = cudaGraphExecMemcpyNodeSetParams1D(hg.exec, hg.out_p, p_out, w.topk_p, kb, d2h) == cudaSuccess;
    if (!ok) {
      cudaGetLastError();
      cudaGraphExecDestroy(hg.exec);
      cudaGraphDestroy(hg.graph);
      hg = HostGraph{};
      hg.failed = true;
      return eager();
    }
  }
  CU(cudaGraphLaunch(hg.exec, st));
  CU(cudaStreamSynchronize(st));
  const int h = *g.h_err;
  if (h) {
    *g.h_err = 0;
    CU(cudaMemsetAsync(g.d_err, 0, sizeof(int), st));
    CU(cudaStreamSynchronize(st));
  }
  return error_status(h);
}

// Upload whose experts come from a reader (the .bin loader); router_w and
// router_b are host memory the caller frees right after, so no host-pointer
// aliases are registered.
int upload_layer_streamed(int layer, const QuantizedWeight* Wg, const QuantizedWeight* Wu,
                          const QuantizedWeight* Wd, const float* router_w, const float* router_b, int E,
                          const ExpertReader& reader) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  return upload_layer(layer, Wg, Wu, Wd, router_w, router_b, E, cudaMemcpyHostToDevice, false, &reader);
}

}  // namespace moe

extern "C" {

int moe_cuda_upload_layer(int layer, const QuantizedWeight* Wg, const QuantizedWeight* Wu,
                          const QuantizedWeight* Wd, const float* router_w, const float* router_b,
                          int E) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  return upload_layer(layer, Wg, Wu, Wd, router_w, router_b, E, cudaMemcpyHostToDevice);
}

int moe_cuda_upload_layer_dev(int layer, const QuantizedWeight* Wg, const QuantizedWeight* Wu,
                              const QuantizedWeight* Wd, const float* router_w,
                              const float* router_b, int E) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  return upload_layer(layer, Wg, Wu, Wd, router_w, router_b, E, cudaMemcpyDeviceToDevice);
}

int moe_cuda_upload_layer_f32(int layer, const float* const* Wg, const float* const* Wu, const float* const* Wd,
                              const float* router_w, const float* router_b, int E, int D, int F, int top_k) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  int rc = ensure_init();
  if (rc) return rc;
  if (g.ep_world > 1) return set_err(MOE_ERR_UNSUPPORTED, "fp32 experts: no expert parallelism");
  if (E <= 0 || D <= 0 || F <= 0 || !Wg || !Wu || !Wd || !router_w)
    return set_err(MOE_ERR_INVALID, "moe_cuda_upload_layer_f32: bad arguments");
  if (top_k < 1 || top_k > 32 || top_k > E || E > 256)
    return set_err(MOE_ERR_UNSUPPORTED, "fp32 experts: top_k %d of E %d (top_k 1..32, E <= 256)", top_k, E);
  for (int e = 0; e < E; ++e)
    if (!Wg[e] || !Wu[e] || !Wd[e]) return set_err(MOE_ERR_INVALID, "expert %d: NULL weight", e);
  host_graphs_reset();
  if (g.layers.count(layer)) moe_cuda_free_layer(layer);
  LayerDev L;
  L.E = E; L.D = D; L.F = F; L.dtype = MOE_DTYPE_F32; L.topk = top_k;
  L.e_begin = 0; L.e_end = E;
  const size_t mb = sizeof(float) * (size_t)F * D;
  L.gq_off = 0;
  L.uq_off = align_up(mb, 128);
  L.dq_off = L.uq_off + align_up(mb, 128);
  L.gs_off = L.us_off = L.ds_off = 0;
  L.expert_stride = align_up(L.dq_off + mb, 128);
  L.bytes = L.expert_stride * (size_t)E;
  if (cudaMalloc((void**)&L.slab, L.bytes) != cudaSuccess)
    return set_err(MOE_ERR_NOMEM, "layer %d: %zu bytes of fp32 expert slabs", layer, L.bytes);
  if (cudaMalloc((void**)&L.router_w, sizeof(float) * (size_t)E * D) != cudaSuccess) {
    cudaFree(L.slab);
    return set_err(MOE_ERR_NOMEM, "layer %d router", layer);
  }
  if (router_b && cudaMalloc((void**)&L.router_b, sizeof(float) * E) != cudaSuccess) {
    cudaFree(L.slab); cudaFree(L.router_w);
    return set_err(MOE_ERR_NOMEM, "layer %d router bias", layer);
  }
  g.layers[layer] = L;
  CU(cudaMemcpy(L.router_w, router_w, sizeof(float) * (size_t)E * D, cudaMemcpyHostToDevice));
  if (router_b) CU(cudaMemcpy(L.router_b, router_b, sizeof(float) * E, cudaMemcpyHostToDevice));
  for (int e = 0; e < E; ++e) {
    uint8_t* base = L.slab + (size_t)e * L.expert_stride;
    CU(cudaMemcpy(base + L.gq_off, Wg[e], mb, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(base + L.uq_off, Wu[e], mb, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(base + L.dq_off, Wd[e], mb, cudaMemcpyHostToDevice));
  }
  return MOE_OK;
}

int moe_cuda_free_layer(int layer) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  auto it = g.layers.find(layer);
  if (it == g.layers.end()) return set_err(MOE_ERR_NOT_INIT, "layer %d was not uploaded", layer);
  cudaDeviceSynchronize();
  host_graphs_reset();
  LayerDev& L = it->second;
  for (auto a = g.alias.begin(); a != g.alias.end();) {
    const uint8_t* d = (const uint8_t*)a->second.dev;
    const bool in_slab = L.slab && d >= L.slab && d < L.slab + L.bytes;
    if (in_slab || d == (const uint8_t*)L.router_w) a = g.alias.erase(a);
    else ++a;
  }
  cudaFree(L.slab); cudaFree(L.router_w);
  if (L.router_b) cudaFree(L.router_b);
  g.layers.erase(it);
  return MOE_OK;
}

size_t moe_cuda_layer_bytes(int layer) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  auto it = g.layers.find(layer);
  return it == g.layers.end() ? 0 : it->second.bytes;
}

int moe_ffn(int layer, const float* x_norm2, float* x_inout, int T, int* topk_idx_out,
            float* topk_p_out, int flags, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const LayerDev* Lp;
  int rc = get_layer(layer, &Lp);
  if (rc) return rc;
  const LayerDev& L = *Lp;
  if (T < 0) return set_err(MOE_ERR_INVALID, "T=%d", T);
  if (T == 0) return MOE_OK;
  if (g.ep_world > 1)
    return set_err(MOE_ERR_INVALID, "expert-parallel run: use moe_ffn_partial + moe_ffn_combine");
  if ((rc = ensure_workspace(T, L.E, L.D, L.F, L.topk))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool host = flags & MOE_FFN_HOST_PTRS;
  const Workspace& w = g.ws;
  const size_t xb = sizeof(float) * (size_t)T * L.D;
  // The kernels of one call on stream s: read xn, update xo in place.
  const bool given = flags & MOE_FFN_GIVEN_TOPK, seq = flags & MOE_FFN_SEQ_RESIDUAL;
  if (given && (!topk_idx_out || !topk_p_out))
    return set_err(MOE_ERR_INVALID, "MOE_FFN_GIVEN_TOPK needs topk_idx_out and topk_p_out (the routing)");
  if (L.dtype == MOE_DTYPE_F32 && (rc = grow(s_hf, sizeof(float) * (size_t)T * L.topk * L.F))) return rc;
  // The combine always runs as its own kernel, after the exact fix-up pass
  // (exact.cu), which recomputes the slots of any token whose activations
  // left the fast kernels' integer range. (Fused into the down epilogue the
  // combine also left the last warp through each row block with T*K dependent
  // loads at the end of the kernel: measured 90 us vs 39 + 6 us.)
  HostOut ho{};     // what the combine publishes to host memory (zero-copy calls below)
  RowCopy zres{};   // zero-copy calls: the residual rows, host -> w.xo, by the routing kernel
  auto enqueue = [&](const float* xn, float* xo, cudaStream_t s) -> int {
    if (L.dtype == MOE_DTYPE_F32) {
      // fp32 experts: router chains + top-k softmax, the fp32 expert FFN, combine
      if (!given) {
        timed("router_logits", s, [&] {
          launch_f32_seq_matmul(xn, L.router_w, L.router_b, w.logits, T, L.E, L.D, s);
        });
        timed("topk_softmax", s, [&] {
          launch_topk_softmax(w.logits, T, L.E, L.topk, w.topk_idx, w.topk_p, s);
        });
      }
      timed("f32_experts", s, [&] { launch_f32_experts(L, xn, w.topk_idx, T, (float*)s_hf.p, w.y, s); });
      timed("combine", s, [&] { launch_combine(w.y, w.topk_p, w.topk_idx, xo, xo, T, L.D, L.topk, s, seq, ho); });
    } else if (use_tensor_cores(L, flags, T)) {
      const int fnt = fused_tile_n(L, T);                 // fused gate/up + down kernel, if used
      const int nt = fnt ? fnt : mma_tile_n(T, L.dtype);
      const float* xres = route_tokens(L, xn, T, nt, s, given, zres.n4 ? &zres : nullptr) ? zres.dst : xo;
      if (T > nt) timed("gather", s, [&] { launch_mma_gather(L, w, T, nt, s); });
      bool ok = true;
      if (fnt) {
        timed("mma_fused", s, [&] { ok = launch_mma_fused(L, w, T, nt, g.d_err, s); });
      } else {
        timed("mma_gateup", s, [&] { ok = launch_mma_gateup(L, w, T, nt, g.d_err, s); });
        if (ok) timed("mma_down", s, [&] { ok = launch_mma_down(L, w, T, nt, w.y, g.d_err, s); });
      }
      if (!ok) return set_err(MOE_ERR_CUDA, "tensor-core launch failed (tensor map or shared memory)");
      timed("exact_fixup", s, [&] {
        launch_exact_fixup(L, xn, w.topk_idx, w.slot_pos, T, w.y, w.xbad, g.sm_count, s);
      });
      timed("combine", s, [&] {
        launch_combine_sorted(w.y, w.slot_pos, w.topk_p, w.topk_idx, xres, xo, T, L.D, L.topk, s, seq, ho);
      });
    } else {
      const float* xres = route_tokens(L, xn, T, 0, s, given, zres.n4 ? &zres : nullptr) ? zres.dst : xo;
      timed("gateup", s, [&] { run_gateup(L, w, T, s); });
      timed("down", s, [&] { run_down(L, w, T, w.y, s); });
      timed("exact_fixup", s, [&] {
        launch_exact_fixup(L, xn, w.topk_idx, nullptr, T, w.y, w.xbad, g.sm_count, s);
      });
      timed("combine", s, [&] { launch_combine(w.y, w.topk_p, w.topk_idx, xres, xo, T, L.D, L.topk, s, seq, ho); });
    }
    CU(cudaGetLastError());
    return MOE_OK;
  };
  const size_t kb = sizeof(int) * (size_t)T * L.topk;
  if (given) {
    // the caller's routing goes where the kernels read it
    const cudaMemcpyKind in_kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    CU(cudaMemcpyAsync(w.topk_idx, topk_idx_out, kb, in_kind, st));
    CU(cudaMemcpyAsync(w.topk_p, topk_p_out, kb, in_kind, st));
  }
  if (host && !st && !g_prof && !given && e2e_graph_on())
    return moe_ffn_host_graph(layer, T, flags, x_norm2, x_inout, topk_idx_out, topk_p_out, xb,
                              sizeof(int) * (size_t)T * L.topk, enqueue);
  const float* xn = x_norm2;
  float* xo = x_inout;
  // Host-pointer call on page-locked buffers: x_inout is read through its
  // mapped address (by the decode routing kernel's spare warps into HBM, else
  // by the combine itself), the combine writes the result there and copies the
  // top-k lists and the error word out, so the call makes one copy (x_norm2
  // in) and one stream synchronisation. Pageable buffers take the copies below.
  if (host) {
    float* zx = (float*)mapped_host_range(x_inout, xb);
    int* zi = topk_idx_out && !given ? (int*)mapped_host_range(topk_idx_out, kb) : nullptr;
    float* zp = topk_p_out && !given ? (float*)mapped_host_range(topk_p_out, kb) : nullptr;
    if (zx && (zi || !topk_idx_out || given) && (zp || !topk_p_out || given)) {
      CU(cudaMemcpyAsync(w.xn, x_norm2, xb, cudaMemcpyHostToDevice, st));
      ho = HostOut{zi, zp, w.topk_idx, w.topk_p, (zi || zp) ? T * L.topk : 0, g.d_err, g.h_err_dev};
      // the residual rows come over the host link once, while the routing
      // chains run, and the combine reads them from HBM
      if ((uintptr_t)zx % 16 == 0 && L.D % 4 == 0) zres = RowCopy{zx, w.xo, (long)T * L.D / 4};
      if ((rc = enqueue(w.xn, zx, st))) return rc;
      return consume_stream_error(st, true);
    }
  }
  if (host) {
    CU(cudaMemcpyAsync(w.xn, x_norm2, xb, cudaMemcpyHostToDevice, st));
    CU(cudaMemcpyAsync(w.xo, x_inout, xb, cudaMemcpyHostToDevice, st));
    xn = w.xn; xo = w.xo;
  }
  if ((rc = enqueue(xn, xo, st))) return rc;
  const cudaMemcpyKind out_kind = host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
  if (topk_idx_out && !given) CU(cudaMemcpyAsync(topk_idx_out, w.topk_idx, kb, out_kind, st));
  if (topk_p_out && !given) CU(cudaMemcpyAsync(topk_p_out, w.topk_p, kb, out_kind, st));
  if (host) {
    CU(cudaMemcpyAsync(x_inout, xo, xb, cudaMemcpyDeviceToHost, st));
    return consume_stream_error(st);
  }
  return MOE_OK;
}

int moe_ffn_partial(int layer, const float* x_norm2, int T, float* y_slots, int* topk_idx_out,
                    float* topk_p_out, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const LayerDev* Lp;
  int rc = get_layer(layer, &Lp);
  if (rc) return rc;
  const LayerDev& L = *Lp;
  if (T < 0) return set_err(MOE_ERR_INVALID, "T=%d", T);
  if (L.dtype == MOE_DTYPE_F32) return set_err(MOE_ERR_UNSUPPORTED, "moe_ffn_partial: fp32 experts (use moe_ffn)");
  if (T == 0) return MOE_OK;
  if ((rc = ensure_workspace(T, L.E, L.D, L.F, L.topk))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const Workspace& w = g.ws;
  const size_t TK = (size_t)T * L.topk;
  if (use_tensor_cores(L, 0, T)) {
    const int nt = mma_tile_n(T, L.dtype);
    route_tokens(L, x_norm2, T, nt, st);
    if (T > nt) timed("gather", st, [&] { launch_mma_gather(L, w, T, nt, st); });
    bool ok = true;
    timed("mma_gateup", st, [&] { ok = launch_mma_gateup(L, w, T, nt, g.d_err, st); });
    if (ok)
      timed("mma_down", st, [&] {
        ok = launch_mma_down(L, w, T, nt, w.y, g.d_err, st);
      });
    if (!ok) return set_err(MOE_ERR_CUDA, "tensor-core launch failed (tensor map or shared memory)");
    timed("unsort", st, [&] { launch_unsort_rows(L, w, T, y_slots, st); });
    timed("exact_fixup", st, [&] {
      launch_exact_fixup(L, x_norm2, w.topk_idx, nullptr, T, y_slots, w.xbad, g.sm_count, st);
    });
  } else {
    CU(cudaMemsetAsync(y_slots, 0, sizeof(float) * TK * L.D, st));
    route_tokens(L, x_norm2, T, 0, st);
    if (L.e_end > L.e_begin) {
      timed("gateup", st, [&] { run_gateup(L, w, T, st); });
      timed("down", st, [&] { run_down(L, w, T, y_slots, st); });
      timed("exact_fixup", st, [&] {
        launch_exact_fixup(L, x_norm2, w.topk_idx, nullptr, T, y_slots, w.xbad, g.sm_count, st);
      });
    }
  }
  if (topk_idx_out) CU(cudaMemcpyAsync(topk_idx_out, w.topk_idx, sizeof(int) * TK, cudaMemcpyDeviceToDevice, st));
  if (topk_p_out) CU(cudaMemcpyAsync(topk_p_out, w.topk_p, sizeof(float) * TK, cudaMemcpyDeviceToDevice, st));
  CU(cudaGetLastError());
  return MOE_OK;
}

int moe_ffn_combine(const float* y_slots, const float* topk_p, float* x_inout, int T, int D,
                    int top_k, void* stream) {
  if (T < 0 || D <= 0 || top_k <= 0) return set_err(MOE_ERR_INVALID, "bad combine shape");
  launch_combine(y_slots, topk_p, nullptr, x_inout, x_inout, T, D, top_k, (cudaStream_t)stream);
  CU(cudaGetLastError());
  return MOE_OK;
}

static inline uint64_t splitmix_at_host(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

void moe_synth_normal_host(uint64_t seed, uint64_t offset, size_t n, float std, float* out) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i) {
    const uint64_t j = offset + (uint64_t)i;
    const double u1 = (double)(splitmix_at_host(seed, 2 * j) >> 11) * 0x1.0p-53;
    const double u2 = (double)(splitmix_at_host(seed, 2 * j + 1) >> 11) * 0x1.0p-53;
    const double z = sqrt(-2.0 * log(1.0 - u1)) * cos(6.283185307179586 * u2);
    out[i] = (float)(z * (double)std);
  }
}

int moe_synth_normal_dev(uint64_t seed, uint64_t offset, size_t n, float std, float* out,
                         void* stream) {
  launch_synth_normal(seed, offset, n, std, out, (cudaStream_t)stream);
  CU(cudaGetLastError());
  return MOE_OK;
}

}  // extern "C"

extern "C" {
int moe_cuda_profile(int enable) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  prof_drain();
  g_prof = enable != 0;
  if (enable) g_prof_acc.clear();
  return MOE_OK;
}

int moe_cuda_profile_read(int max_kernels, char* names, int name_len, double* total_ms, long* launches) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  prof_drain();
  int i = 0;
  for (auto& kv : g_prof_acc) {
    if (i >= max_kernels) break;
    snprintf(names + (size_t)i * name_len, (size_t)name_len, "%s", kv.first.c_str());
    total_ms[i] = kv.second.first;
    launches[i] = kv.second.second;
    ++i;
  }
  return i;
}
}  // extern "C"

// ---------------------------------------------------------------------------
// expert parallelism: dispatch fused into the routing kernel, exchange of the
// slot rows fused into the down GEMM (buffer layout: EpView in kernels.cuh)
// ---------------------------------------------------------------------------
namespace moe {
struct EpCtx {
  bool ready = false, connected = false;
  int cap_tokens = 0, D = 0, K = 0, world = 0;
  uint8_t* buf = nullptr;
  size_t xact_off = 0, xsum_off = 0, idx_off = 0, p_off = 0, y_off = 0, xf_off = 0, xflag_off = 0;
  size_t parity_bytes = 0;
  void* peer_base[kEpMaxRanks] = {};
  uint8_t** d_base = nullptr;                // device array of the peers' bases
  cudaIpcMemHandle_t own{};                  // this rank's handle (ep_setup)
  unsigned long long seq = 0;
};
static EpCtx g_ep;

static void ep_release() {
  for (int p = 0; p < kEpMaxRanks; ++p)
    if (g_ep.peer_base[p] && g_ep.peer_base[p] != g_ep.buf) cudaIpcCloseMemHandle(g_ep.peer_base[p]);
  if (g_ep.buf) cudaFree(g_ep.buf);
  if (g_ep.d_base) cudaFree(g_ep.d_base);
  g_ep = EpCtx{};
}
static void ep_shutdown_hook() { ep_release(); }

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Time limit of the device-side waits on the other ranks' flags (dispatch in
// the routing kernel, combine in ep_combine): MOE_EP_WAIT_MS, default 200 ms.
// Ranks must enter each moe_ffn_ep call within that time of one another; a
// wait that runs out reports MOE_ERR_CUDA through moe_cuda_check_status.
static unsigned long long ep_wait_ns() {
  static long long ms = -1;
  if (ms < 0) {
    const char* e = getenv("MOE_EP_WAIT_MS");
    ms = e && atoll(e) > 0 ? atoll(e) : 200;
  }
  return (unsigned long long)ms * 1000000ull;
}
}  // namespace moe

extern "C" {

#ifdef MOE_TIMELINE
// Timeline build only: copy out (and optionally reset) the per-kernel
// [first start, last end] globaltimer table, kTlCount x 2 values.
int moe_debug_q4_trace(long long* out) {
  CU(cudaDeviceSynchronize());
  moe::q4_trace_read(out);
  return MOE_OK;
}

int moe_debug_fused_trace(unsigned long long* out) {
  CU(cudaDeviceSynchronize());
  moe::fz_trace_read(out);
  return MOE_OK;
}

int moe_debug_timeline(unsigned long long* out, int reset) {
  CU(cudaDeviceSynchronize());
  unsigned long long t[2 * kTlCount];
  for (int i = 0; i < kTlCount; ++i) { t[2 * i] = ~0ull; t[2 * i + 1] = 0; }
  moe::tl_io_router(t, reset);
  moe::tl_io_moe_mma(t, reset);
  moe::tl_io_ep(t, reset);
  moe::tl_io_moe_fused(t, reset);
  if (out) memcpy(out, t, sizeof(t));
  return MOE_OK;
}
#endif

int moe_cuda_ep_setup(int max_tokens_local, int D, int top_k, void* ipc_handle_out) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  int rc = ensure_init();
  if (rc) return rc;
  const int W = g.ep_world;
  if (W < 2) return set_err(MOE_ERR_INVALID, "moe_cuda_ep_setup needs an expert-parallel group (ep_world > 1)");
  if (W > kEpMaxRanks) return set_err(MOE_ERR_UNSUPPORTED, "at most %d ranks", kEpMaxRanks);
  if (max_tokens_local <= 0 || D <= 0 || top_k <= 0 || !ipc_handle_out)
    return set_err(MOE_ERR_INVALID, "moe_cuda_ep_setup: bad arguments");
  ep_release();
  const size_t TA = (size_t)W * max_tokens_local;          // tokens of all ranks
  size_t o = 0;
  g_ep.xact_off = o;  o = align256(o + TA * 2 * D);
  g_ep.xsum_off = o;  o = align256(o + TA * 4);
  g_ep.idx_off = o;   o = align256(o + TA * top_k * 4);
  g_ep.p_off = o;     o = align256(o + TA * top_k * 4);
  g_ep.y_off = o;     o = align256(o + (size_t)max_tokens_local * top_k * D * 4);
  g_ep.xf_off = o;    o = align256(o + (size_t)max_tokens_local * D * 4);
  g_ep.xflag_off = o; o = align256(o + (2 + (size_t)max_tokens_local) * 4);
  g_ep.parity_bytes = o;
  const size_t bytes = kEpHeader + 2 * o;
  if (cudaMalloc((void**)&g_ep.buf, bytes) != cudaSuccess)
    return set_err(MOE_ERR_NOMEM, "expert-parallel buffers (%zu bytes)", bytes);
  CU(cudaMemset(g_ep.buf, 0, bytes));
  cudaIpcMemHandle_t h;
  CU(cudaIpcGetMemHandle(&h, g_ep.buf));
  memcpy(ipc_handle_out, &h, sizeof(h));
  g_ep.own = h;
  g_ep.cap_tokens = max_tokens_local; g_ep.D = D; g_ep.K = top_k; g_ep.world = W;
  g_ep.ready = true;
  return MOE_OK;
}

int moe_cuda_ep_connect(const void* ipc_handles) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  if (!g_ep.ready) return set_err(MOE_ERR_NOT_INIT, "moe_cuda_ep_setup has not been called");
  if (!ipc_handles) return set_err(MOE_ERR_INVALID, "moe_cuda_ep_connect: null handles");
  const int W = g_ep.world;
  const cudaIpcMemHandle_t* hs = (const cudaIpcMemHandle_t*)ipc_handles;
  std::vector<uint8_t*> base(W);
  for (int p = 0; p < W; ++p) {
    // this rank's own buffer, and any entry holding this rank's own handle
    // (a loopback group in one process, whose waits on the other entries
    // can only expire: used to test the bounded waits on one GPU)
    if (p == g.ep_rank || memcmp(&hs[p], &g_ep.own, sizeof(g_ep.own)) == 0) {
      g_ep.peer_base[p] = g_ep.buf;
    } else if (!g_ep.peer_base[p]) {
      void* ptr = nullptr;
      CU(cudaIpcOpenMemHandle(&ptr, hs[p], cudaIpcMemLazyEnablePeerAccess));
      g_ep.peer_base[p] = ptr;
    }
    base[p] = (uint8_t*)g_ep.peer_base[p];
  }
  if (!g_ep.d_base) CU(cudaMalloc((void**)&g_ep.d_base, sizeof(uint8_t*) * W));
  CU(cudaMemcpy(g_ep.d_base, base.data(), sizeof(uint8_t*) * W, cudaMemcpyHostToDevice));
  g_ep.connected = true;
  return MOE_OK;
}

int moe_ffn_ep(int layer, const float* x_norm2, int T_local, float* x_inout, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const LayerDev* Lp;
  int rc = get_layer(layer, &Lp);
  if (rc) return rc;
  const LayerDev& L = *Lp;
  if (!g_ep.connected) return set_err(MOE_ERR_NOT_INIT, "moe_cuda_ep_connect has not been called");
  if (T_local < 0 || T_local > g_ep.cap_tokens || L.D != g_ep.D || L.topk != g_ep.K)
    return set_err(MOE_ERR_INVALID, "moe_ffn_ep: T_local=%d exceeds the buffers (%d) or the layer shape differs",
                   T_local, g_ep.cap_tokens);
  const int W = g_ep.world, T = T_local * W;
  if (!use_tensor_cores(L, MOE_FFN_FORCE_GEMM, T))
    return set_err(MOE_ERR_UNSUPPORTED, "moe_ffn_ep needs the tensor-core path (Q8/Q4, D and F multiples of 128)");
  if (T_local == 0) return MOE_OK;
  if (!decode_route_supported(L, T, x_norm2))
    return set_err(MOE_ERR_UNSUPPORTED,
                   "moe_ffn_ep: %d routed slots per step over all ranks (at most 2048), or unaligned input",
                   T * L.topk);
  if ((rc = ensure_workspace(T, L.E, L.D, L.F, L.topk))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned long long seq = ++g_ep.seq;
  const size_t par = (seq & 1) ? g_ep.parity_bytes : 0;
  EpView ep;
  ep.base = g_ep.d_base; ep.base_local = g_ep.buf;
  ep.world = W; ep.rank = g.ep_rank; ep.T_local = T_local; ep.seq = seq;
  ep.xact_off = kEpHeader + par + g_ep.xact_off; ep.xsum_off = kEpHeader + par + g_ep.xsum_off;
  ep.idx_off = kEpHeader + par + g_ep.idx_off;   ep.p_off = kEpHeader + par + g_ep.p_off;
  ep.y_off = kEpHeader + par + g_ep.y_off;
  ep.xf_off = kEpHeader + par + g_ep.xf_off;     ep.xflag_off = kEpHeader + par + g_ep.xflag_off;
  ep.wait_ns = ep_wait_ns();
  // the expert kernels read all ranks' tokens from the exchange buffers
  Workspace w = g.ws;
  w.xact = g_ep.buf + ep.xact_off;
  w.xsum = (int*)(g_ep.buf + ep.xsum_off);
  w.topk_idx = (int*)(g_ep.buf + ep.idx_off);
  w.topk_p = (float*)(g_ep.buf + ep.p_off);
  w.cap_T = std::min(g.ws.cap_T, W * g_ep.cap_tokens);     // rows the tensor maps may cover
  const int fnt = fused_tile_n(L, T);
  const int nt = fnt ? fnt : mma_tile_n(T, L.dtype);
  timed("route_dispatch", st, [&] {
    launch_decode_route(L, g.ws, x_norm2, T_local, nt, g.ws.route_counter, g.d_err, st, &ep);
  });
  if (T > nt) timed("gather", st, [&] { launch_mma_gather(L, w, T, nt, st); });
  bool ok = true;
  if (fnt) {
    timed("mma_fused_ep", st, [&] { ok = launch_mma_fused(L, w, T, nt, g.d_err, st, &ep); });
  } else {
    timed("mma_gateup", st, [&] { ok = launch_mma_gateup(L, w, T, nt, g.d_err, st); });
    if (ok)
      timed("mma_down_ep", st, [&] {
        ok = launch_mma_down(L, w, T, nt, w.y, g.d_err, st, &ep);
      });
  }
  if (!ok) return set_err(MOE_ERR_CUDA, "tensor-core launch failed (tensor map or shared memory)");
  // exact recomputation of out-of-range tokens' slots; raises the combine flags
  timed("exact_fixup_ep", st, [&] {
    launch_exact_fixup(L, nullptr, w.topk_idx, nullptr, T, nullptr, w.xbad, g.sm_count, st, &ep);
  });
  timed("ep_combine", st, [&] { launch_ep_combine(ep, x_inout, x_inout, L.D, L.topk, g.d_err, st); });
  CU(cudaGetLastError());
  return MOE_OK;
}

}  // extern "C"
