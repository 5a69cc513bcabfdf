// kernels.cuh — kernel launch interfaces shared by the .cu files of libmoe_cuda.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace moe {

// Device-resident layer (one expert-parallel shard of one MoE layer).
// Each local expert owns one slab of `expert_stride` bytes:
//   [gate q | up q | down q | gate s | up s | down s], parts 128 B aligned.
// dtype 2 (Q8), 3 (Q4) or 0 (fp32 experts: gate [F][D], up [F][D] and down
// [D][F] floats at gq_off, uq_off, dq_off; no scales).
struct LayerDev {
  int E = 0, D = 0, F = 0, dtype = 0, topk = 8;
  int e_begin = 0, e_end = 0;         // this rank's experts [e_begin, e_end)
  int gu_rb = 0, d_rb = 0;            // row bytes: gate/up (D or D/2), down (F or F/2)
  uint8_t* slab = nullptr;
  size_t expert_stride = 0;
  size_t gq_off = 0, uq_off = 0, dq_off = 0, gs_off = 0, us_off = 0, ds_off = 0;
  float* router_w = nullptr;          // [E][D]
  float* router_b = nullptr;          // [E] or null
  size_t bytes = 0;
};

// Source of one local expert's slab image for a streamed upload: fill writes
// the six parts at the LayerDev offsets (gq_off .. ds_off) into `img`
// (expert_stride bytes of host memory) and returns false on a read error,
// after setting the library's error message.
struct ExpertReader {
  bool (*fill)(void* ctx, int e, const LayerDev& L, uint8_t* img);
  void* ctx;
};

// Per-call scratch of moe_ffn (capacity for up to cap_T tokens).
struct Workspace {
  int cap_T = 0, cap_D = 0, cap_E = 0, cap_F = 0, cap_K = 0;
  float* logits = nullptr;    // [T][E]
  int* topk_idx = nullptr;    // [T][K]
  float* topk_p = nullptr;    // [T][K]
  int* route = nullptr;       // n_active | active[E] | exp_off[E+1] | slot_list[T*K]
  uint8_t* xact = nullptr;    // token activations, 2*D bytes per token
  int* xsum = nullptr;        // [T]  Σ activation (Q4 zero-point correction)
  int* xsum_s = nullptr;      // [T*K] Σ activation of each expert-sorted slot's token (gathered rows)
  uint8_t* hact = nullptr;    // slot activations, 2*F bytes per slot
  int* hsum = nullptr;        // [T*K]
  float* y = nullptr;         // [T*K][D]
  int* route_counter = nullptr;  // arrival counter of the fused routing kernel (kept zero)
  uint8_t* xs0 = nullptr;     // expert-sorted token activations, plane 0 [T*K][D]
  uint8_t* xs1 = nullptr;     //   plane 1 (Q8 high limb)
  uint8_t* hs0 = nullptr;     // expert-sorted down-projection inputs [T*K][F]
  uint8_t* hs1 = nullptr;
  int* slot_pos = nullptr;    // [T*K] slot -> expert-sorted row
  float* xn = nullptr;        // staging for host-pointer calls [T][D]
  float* xo = nullptr;        // [T][D]
  int* fused_ctr = nullptr;   // fused decode kernel: work, arrival, per-tile completion (kept zero)
  // Per-call range flags of the exact fix-up pass, [2 + cap_T] ints kept zero
  // between calls: [0] any token flagged, [1] the pass's arrival counter,
  // [2 + t] token t had an activation (x, or h of one of its slots) outside
  // the fast kernels' integer range. Null: kernels report kErrRange instead.
  int* xbad = nullptr;
};

// Expert-parallel exchange buffers. Every rank allocates the same layout
// (CUDA IPC-shared): at offset 0 the dispatch flags [kEpMaxRanks] u64 and the
// combine flags [kEpMaxRanks] u64 (rank r raises entry r; values are call
// sequence numbers, so they only grow), then an int arrival counter of the
// down kernel (local, kept zero); then two parities of data, alternate calls
// using alternate parities:
//   xact [world*T_local][2*D] u8   truncated activations of every rank's tokens
//   xsum [world*T_local] int       their Σ (Q4 zero point)
//   idx, p [world*T_local*K]       every rank's top-k choice and weight
//   y [T_local*K][D] f32           this rank's slot rows, stored by the owners
//                                  of the slots' experts
//   xf [T_local][D] f32            this rank's MoE inputs as given (local
//                                  stores; the exact fix-up pass of the
//                                  experts' owners reads them over NVLink)
//   xflag [2 + T_local] int        [0] and [2 + t]: equal to the low 32 bits
//                                  of seq when some token / token t of this
//                                  rank had an activation outside the fast
//                                  kernels' range in this call
// base[] holds the peers' mappings (own buffer at base[rank]); the *_off
// fields point into this call's parity.
constexpr int kEpMaxRanks = 64;
constexpr size_t kEpDispatchFlags = 0, kEpCombineFlags = 8 * kEpMaxRanks, kEpCounter = 16 * kEpMaxRanks;
constexpr size_t kEpHeader = 16 * kEpMaxRanks + 256;
struct EpView {
  uint8_t* const* base = nullptr;   // device array [world]
  uint8_t* base_local = nullptr;    // == base[rank]
  int world = 0, rank = 0, T_local = 0;
  unsigned long long seq = 0;
  unsigned long long wait_ns = 0;   // limit of each wait on the other ranks' flags
  size_t xact_off = 0, xsum_off = 0, idx_off = 0, p_off = 0, y_off = 0, xf_off = 0, xflag_off = 0;
};

#ifdef __CUDACC__
}  // namespace moe
#include "pipeline.cuh"
namespace moe {
// One thread, once the rank's y-row stores of this call are complete: raise
// this rank's combine flag (entry ep.rank, value ep.seq) at every rank,
// starting with itself, after a system fence (release), so a rank that sees
// the flag sees the rows.
__device__ __forceinline__ void ep_raise_combine(const EpView& ep) {
  __threadfence_system();
  for (int i = 0; i < ep.world; ++i) {
    const int p = (ep.rank + i) % ep.world;
    uint8_t* pb = reinterpret_cast<uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(ep.base) + p));
    st_release_sys(reinterpret_cast<unsigned long long*>(pb + kEpCombineFlags) + ep.rank, ep.seq);
  }
}
#endif

struct RouteView {
  int* n_active; int* active; int* exp_off; int* slot_list;
};
// tile table after the routing lists: n_tiles | tile_u[m] | tile_j0[m] | tile_n[m]
struct TileView { const int* n; const int* u; const int* j0; const int* cnt; };
__host__ __device__ inline TileView tile_view(const int* route, int E, int TK, int m) {
  const int* t = route + 2 + 2 * E + TK;
  return {t, t + 1, t + 1 + m, t + 1 + 2 * m};
}

__host__ __device__ inline RouteView route_view(int* route, int E) {
  RouteView r;
  r.n_active = route;
  r.active = route + 1;
  r.exp_off = route + 1 + E;
  r.slot_list = route + 2 + 2 * E;
  return r;
}

// ---- launchers (all asynchronous on `st`) ----
// xact planes from fp32 rows: Q8 -> [lo K][hi K] per row, Q4 -> permuted K
// bytes per row + rowsum. Sets err bit kErrRange on out-of-range values.
// mma_layout: Q4 activations in the tensor-core order (q4_mma_pos)
// flags: per-token range flags (range_fail in common.cuh) instead of kErrRange.
// mark != 0: an out-of-range activation stores mark into *err instead (the
// fast GEMV of the same call compares it), so *err needs no clearing
void launch_quantize_act(const float* x, int M, int K, int dtype, uint8_t* act,
                         int act_stride, int* asum, int* err, cudaStream_t st,
                         int mma_layout = 0, int* flags = nullptr, int mark = 0);
// C[m][n] = sequential fp32 Σ_k A[m][k] W[n][k] (+ b[n]).
void launch_f32_seq_matmul(const float* A, const float* W, const float* b,
                           float* C, int M, int N, int K, cudaStream_t st);
void launch_topk_softmax(const float* logits, int T, int E, int K, int* idx,
                         float* p, cudaStream_t st);
// nt > 0: also the tensor-core tile table (nt slots per tile) and slot_pos
void launch_route_build(const int* idx, int T, int K, int e_begin, int e_end,
                        int* route, int E_local, int* hsum, int nt, int* slot_pos,
                        cudaStream_t st);
int route_max_tiles(int TK, int E_local, int nt);
// the same lists built by 1024 threads (any slot count, E_local <= kRouteBuildMaxE)
constexpr int kRouteBuildMaxE = 256;
void launch_route_build_multi(const int* idx, int T, int K, int e_begin, int E_local, int* route,
                              int* hsum, int nt, int* slot_pos, cudaStream_t st);
// Fast warp GEMV over n_mat matrices: C[mat][m][n]. Returns false if the
// shape has no fast-path geometry (caller uses the generic kernel). With A
// (the fp32 activations), flag and mark (launch_quantize_act's err word and
// mark): when *flag == mark the kernel computes every output exactly from A
// instead, so the result is the reference's for any activation magnitude.
bool launch_gemv(int dtype, const uint8_t* const* Wq, const float* const* Ws,
                 int n_mat, bool ptr_arrays_on_device, int N, int K,
                 const uint8_t* act, int act_stride, const int* asum, int M,
                 float* C, cudaStream_t st, const float* A = nullptr, const int* flag = nullptr,
                 int mark = 0);
// a fresh nonzero mark per call (thread-safe)
int next_range_mark();
// Exact kernel for any shape and activation magnitude (one thread per output,
// int32 truncation, wrapping dot).
void launch_gemv_generic(int dtype, const float* A, const uint8_t* Wq,
                         const float* Ws, float* C, int M, int N, int K,
                         cudaStream_t st);
bool fast_geometry_ok(int dtype, int K);
void launch_gateup(const LayerDev& L, const Workspace& ws, int T, int* err,
                   cudaStream_t st);
// down projection: slot rows y[s][D] for launch_combine
void launch_down(const LayerDev& L, const Workspace& ws, int T, float* y, cudaStream_t st);
// Exact fix-up pass (exact.cu): when flags[0] is set, recomputes y of every
// slot of each flagged token whose expert is local, with int32 activations
// of any magnitude, into row slot_pos[s] (or s when slot_pos is null) of y;
// the last CTA clears the flags. A no-op launch when nothing was flagged.
// ep != null (expert parallel; T = all ranks' tokens, idx = all ranks' top-k):
// tokens are also flagged by their home rank's xflag, their inputs are read
// from its xf, y rows go to its y buffer, and the last CTA raises this rank's
// combine flags at every rank.
void launch_exact_fixup(const LayerDev& L, const float* xn, const int* idx, const int* slot_pos, int T,
                        float* y, int* flags, int sm_count, cudaStream_t st, const EpView* ep = nullptr);
// What a combine kernel also copies into page-locked host memory for a
// host-pointer call, so that call needs no device-to-host copies: the top-k
// lists (n = T*K entries; null destinations are skipped) and the call's
// error word. The combine runs after every other kernel of the call has
// completed, so the values it copies are final.
struct HostOut {
  int* idx; float* p; const int* idx_src; const float* p_src; int n;
  const int* err_src; int* err;
};
// grid-strided over the combine's threads (q = global thread index)
__device__ __forceinline__ void publish_host(const HostOut& h, long q, long nthreads) {
  for (long i = q; i < h.n; i += nthreads) {
    if (h.idx) h.idx[i] = h.idx_src[i];
    if (h.p) h.p[i] = h.p_src[i];
  }
  if (q == 0 && h.err) *h.err = *reinterpret_cast<const volatile int*>(h.err_src);
}
// seq_residual: out = ((xres + p0 y0) + p1 y1) + ... (model.c:188) instead of
// xres + (((0 + p0 y0) + p1 y1) + ...) (test_model_trace.c:513,517)
void launch_combine(const float* y, const float* p, const int* idx, const float* xres,
                    float* out, int T, int D, int K, cudaStream_t st, bool seq_residual = false,
                    const HostOut& ho = HostOut{});
// fp32 experts (f32_experts.cu): h [T*K][F], y [T*K][D] (slot rows)
void launch_f32_experts(const LayerDev& L, const float* xn, const int* idx, int T, float* h, float* y,
                        cudaStream_t st);
void launch_quantize_rowwise(int dtype, const float* W, int rows, int cols,
                             void* q, float* s, cudaStream_t st);
void launch_synth_normal(uint64_t seed, uint64_t offset, size_t n, float std,
                         float* out, cudaStream_t st);
void launch_zero_fill(float* C, size_t n, cudaStream_t st);

}  // namespace moe

namespace moe {
// moe_mma.cu: tcgen05 grouped GEMMs over the routed experts
bool mma_supported(const LayerDev& L);
int mma_tile_n(int T, int dtype);
void launch_mma_gather(const LayerDev& L, const Workspace& ws, int T, int nt, cudaStream_t st);
bool launch_mma_gateup(const LayerDev& L, const Workspace& ws, int T, int nt, int* err, cudaStream_t st);
// ep != null: expert-parallel mode, each slot row is stored into the y buffer
// of the rank owning its token, and the last CTA raises this rank's combine
// flag at every peer
bool launch_mma_down(const LayerDev& L, const Workspace& ws, int T, int nt, float* ys, int* err, cudaStream_t st,
                     const EpView* ep = nullptr);
// moe_fused.cu: Q8 decode gate/up + down in one persistent kernel
constexpr int kFusedMaxTiles = 256;
// tile width the fused kernel would use for T tokens (16 or 32), 0 = not used
int fused_tile_n(const LayerDev& L, int T);
bool launch_mma_fused(const LayerDev& L, const Workspace& ws, int T, int nt, int* err, cudaStream_t st,
                      const EpView* ep = nullptr);
void launch_combine_sorted(const float* ys, const int* slot_pos, const float* p, const int* idx,
                           const float* xres, float* out, int T, int D, int K, cudaStream_t st,
                           bool seq_residual = false, const HostOut& ho = HostOut{});
void launch_unsort_rows(const LayerDev& L, const Workspace& ws, int T, float* y_slots, cudaStream_t st);
}  // namespace moe

namespace moe {
// router.cu: decode routing prologue in one launch
bool decode_route_supported(const LayerDev& L, int T, const float* x);
// ep != null: T = this rank's tokens; their activations and top-k go to every
// rank's buffers, and the routing lists cover all ranks' tokens (after a
// bounded wait on the dispatch flags)
// res: a copy the routing kernel's spare warps make while the chains run
// (n4 16-byte words from src to dst), e.g. a call's residual rows from
// page-locked host memory into the device workspace
struct RowCopy { const float* src; float* dst; long n4; };
void launch_decode_route(const LayerDev& L, const Workspace& ws, const float* x, int T, int nt,
                         int* counter, int* err, cudaStream_t st, const EpView* ep = nullptr,
                         const RowCopy* res = nullptr);
}  // namespace moe

namespace moe {
// ep.cu: the combine of the expert-parallel exchange (waits on the ranks'
// combine flags, then the k-ordered combine of this rank's tokens)
void launch_ep_combine(const EpView& ep, const float* xres, float* out, int D, int K, int* err,
                       cudaStream_t st);
}  // namespace moe
