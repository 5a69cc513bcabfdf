// router.cu — the decode-regime routing prologue in one launch.
//
// grid = (E/8 expert blocks) x (ceil(T/8) token blocks), 512 threads. Each
// CTA bulk-copies its 8 router rows and 8 token rows into shared memory once
// (1-D bulk async copies in four column chunks, one mbarrier each), then each
// of 64 threads runs one exact sequential fp32 chain
// logits[t][e] = Σ_k x[t][k]·W[e][k] (+b[e]) in k order
// (test_model_trace.c:213-227, :465-468) straight from shared memory, while
// the other warps truncate the CTA's slice of the token activations for the
// expert kernels (kernels.c:66 / :113). The last CTA to finish (arrival
// counter) then does, for all tokens: top-k (topk_desc, :275-288, as K warp
// arg-max rounds over per-lane sorted candidates), the
// top-k softmax (:481-487), and the routing lists, tensor-core tile table and
// slot -> expert-sorted-row map. That phase keeps its tables in shared memory
// (per-expert counts by shared atomics, one warp-shuffle scan over experts)
// and writes them out with all threads: a single thread issuing hundreds of
// scattered global stores was measured at ~15 us per table.
#include "common.cuh"
#include "kernels.cuh"
#include "pipeline.cuh"

namespace moe {
namespace rt {

// 8 experts x 8 tokens per CTA: two warps of chains per SM. Each k step of a
// chain warp costs about two shared-memory wavefronts (its x and W loads), and
// the SM serves one wavefront per cycle, so with four chain warps (16 tokens)
// the chains ran at ~8 cycles per dependent add against ~4.9 with two.
constexpr int kE = 8, kT = 8, kThreads = 512, kChainThreads = kE * kT, kChunks = 4;
constexpr int kMaxTK = 2048;    // T*K handled by the last CTA (decode and EP-gathered sizes)
constexpr int kMaxE = 256;
constexpr int kMaxTiles = kMaxTK / 16 + kMaxE + 1;

struct Args {
  const float* x; const float* W; const float* b;
  int T, E, D, K;
  float* logits; int* idx; float* p;
  int* route; int e_begin, E_local; int* hsum; int nt, max_tiles; int* slot_pos;
  uint8_t* xact; int* xsum; int q4_mma;
  int* counter; int* err;
  int* flags;              // per-token range flags (range_fail) or null
  RowCopy res;             // copied by the non-chain warps of all CTAs (n4 = 0: none)
  int ep_on; EpView ep;    // expert parallel: dispatch this rank's tokens, route all ranks' tokens
};

__device__ __forceinline__ uint8_t* peer_base(const EpView& ep, int p) {
  return reinterpret_cast<uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(ep.base) + p));
}

template <int DT>
__global__ void __launch_bounds__(kThreads) decode_route_kernel(const Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int pitch = a.D + 4;                                   // floats; padding spreads banks
  float* sw = reinterpret_cast<float*>(smem);                  // [kE][pitch]
  float* sx = sw + kE * pitch;                                 // [kT][pitch]
  __shared__ uint64_t bar[kChunks];
  __shared__ int s_last;
  const int e0 = blockIdx.x * kE, t0 = blockIdx.y * kT;
  const int ne = min(kE, a.E - e0), nt = min(kT, a.T - t0);
  const int tid = threadIdx.x;
  const int dc = a.D / kChunks;                                // columns per chunk
  MOE_TL_START(kTlRoute);

  // the rows arrive in kChunks column chunks, each on its own barrier, so the
  // chains start on chunk 0 while the rest is still in flight. The copies
  // are issued by all lanes of warp 0 (one thread issuing them one after
  // another measured ~35 ns per copy).
  if (tid < 32) {
    if (tid == 0) {
      for (int c = 0; c < kChunks; ++c) mbar_init(&bar[c], 1);
      fence_mbar_init();
      for (int c = 0; c < kChunks; ++c) mbar_arrive_expect_tx(&bar[c], (uint32_t)((ne + nt) * dc * 4));
    }
    __syncwarp();
    // the router rows are constant: they go out before the wait for the
    // previous kernel (dependent launch); the token rows after it
    for (int q = tid; q < kChunks * ne; q += 32) {
      const int c = q / ne, i = q % ne;
      bulk_g2s(sw + i * pitch + c * dc, a.W + (size_t)(e0 + i) * a.D + c * dc, dc * 4, &bar[c]);
    }
    pdl_wait();
    for (int q = tid; q < kChunks * nt; q += 32) {
      const int c = q / nt, i = q % nt;
      bulk_g2s(sx + i * pitch + c * dc, a.x + (size_t)(t0 + i) * a.D + c * dc, dc * 4, &bar[c]);
    }
  }
  pdl_wait();
  pdl_launch();
  __syncthreads();
  // A timed-out copy flags the call as failed; the CTA still reports its
  // arrival below so the arrival counter stays consistent for later calls.
  bool ok = true;

  if (tid < kChainThreads) {
    // ---- exact sequential chain: one (token, expert) per thread ----
    const int tt = tid / kE, ee = tid % kE;
    const bool mine = tt < nt && ee < ne;
    const float* xr = sx + tt * pitch;
    const float* wr = sw + ee * pitch;
    float acc = 0.0f;
    for (int c = 0; c < kChunks; ++c) {
      if (!mbar_wait(&bar[c], 0, kWaitNs)) { ok = false; break; }
      if (!mine) continue;
      // 16-k register blocks: the block's products, the next block's loads
      // (their latency overlaps the adds), then the 16 dependent adds in k order
      const float* xc = xr + c * dc;
      const float* wc = wr + c * dc;
      const int nb = dc / 16;
      float4 xb[4], wb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { xb[i] = lds4(xc + 4 * i); wb[i] = lds4(wc + 4 * i); }
      for (int blk = 0; blk < nb; ++blk) {
        float pr[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pr[4 * i] = mul_rn(xb[i].x, wb[i].x);
          pr[4 * i + 1] = mul_rn(xb[i].y, wb[i].y);
          pr[4 * i + 2] = mul_rn(xb[i].z, wb[i].z);
          pr[4 * i + 3] = mul_rn(xb[i].w, wb[i].w);
        }
        const int nxt = blk + 1 < nb ? blk + 1 : blk;
#pragma unroll
        for (int i = 0; i < 4; ++i) { xb[i] = lds4(xc + 16 * nxt + 4 * i); wb[i] = lds4(wc + 16 * nxt + 4 * i); }
#pragma unroll
        for (int i = 0; i < 16; ++i) acc = add_rn(acc, pr[i]);
      }
    }
    if (ok && mine) {
      if (a.b) acc = fadd(acc, __ldg(a.b + e0 + ee));
      a.logits[(size_t)(t0 + tt) * a.E + e0 + ee] = acc;
    }
  } else {
    // ---- truncated activations: this CTA's column slice of its tokens ----
    const int q0 = tid - kChainThreads, nq = kThreads - kChainThreads;
    // wait only for the chunks holding this CTA's column slice (the Q4 Σa of
    // CTA 0 needs every column), so these warps do not poll beside the chains
    const int cs0 = (int)((long)a.D * blockIdx.x / gridDim.x), cs1 = (int)((long)a.D * (blockIdx.x + 1) / gridDim.x);
    const bool all = DT == 4 && blockIdx.x == 0;
    const int cf = all ? 0 : cs0 / dc, cl = all ? kChunks - 1 : (cs1 - 1) / dc;
    for (int c = cf; c <= cl && cs1 > cs0; ++c)
      if (!mbar_wait(&bar[c], 0, kWaitNs)) { ok = false; break; }
    // expert parallel: the activations go to every rank's xact (rows of this
    // rank's tokens), starting with the next rank so the links share the load
    const int ndst = a.ep_on ? a.ep.world : 1;
    for (int di = 0; ok && di < ndst; ++di) {
      uint8_t* xact = a.xact;
      int* xsum = a.xsum;
      if (a.ep_on) {
        uint8_t* pb = peer_base(a.ep, (a.ep.rank + 1 + di) % a.ep.world);
        xact = pb + a.ep.xact_off + (size_t)a.ep.rank * a.ep.T_local * 2 * a.D;
        xsum = reinterpret_cast<int*>(pb + a.ep.xsum_off) + a.ep.rank * a.ep.T_local;
      }
      const int c0 = (int)((long)a.D * blockIdx.x / gridDim.x);
      const int c1 = (int)((long)a.D * (blockIdx.x + 1) / gridDim.x);
      const int w = c1 - c0;
      for (int q = q0; q < nt * w; q += nq) {
        const int t = q / w, k = c0 + q % w;
        const int v = trunc_scale(sx[t * pitch + k], DT == 8 ? 127.0f : 7.0f);
        uint8_t* ar = xact + (size_t)(t0 + t) * 2 * a.D;
        bool bad;
        if (DT == 8) {
          bad = v < -32768 || v > 32767;
          ar[k] = (uint8_t)(v & 0xFF);
          ar[a.D + k] = (uint8_t)((v >> 8) & 0xFF);
        } else {
          bad = v < -128 || v > 127;
          ar[a.q4_mma ? q4_mma_pos(k) : q4_act_pos(k)] = (uint8_t)(v & 0xFF);
        }
        if (di == 0) {
          if (a.ep_on) {
            // the MoE input as given, for the experts' owners' exact fix-up,
            // and this rank's out-of-range marks (this call's sequence number)
            reinterpret_cast<float*>(a.ep.base_local + a.ep.xf_off)[(size_t)(t0 + t) * a.D + k] =
                sx[t * pitch + k];
            if (bad) {
              int* xflag = reinterpret_cast<int*>(a.ep.base_local + a.ep.xflag_off);
              xflag[2 + t0 + t] = (int)a.ep.seq;
              xflag[0] = (int)a.ep.seq;
            }
          } else if (bad) {
            range_fail(a.err, a.flags, t0 + t);
          }
        }
      }
      if (DT == 4 && blockIdx.x == 0) {       // Σ activation per token (Q4 zero point)
        for (int t = q0 / 32; t < nt; t += nq / 32) {
          int sacc = 0;
          for (int k = q0 % 32; k < a.D; k += 32) sacc += trunc_scale(sx[t * pitch + k], 7.0f);
          sacc = warp_sum(sacc);
          if ((q0 & 31) == 0) xsum[t0 + t] = sacc;
        }
      }
    }
  }
  if (tid >= kChainThreads && a.res.n4 > 0) {
    // spare warps: the caller's extra copy, spread over every CTA (all its
    // loads are independent, so its latency overlaps the chains)
    const int nq = kThreads - kChainThreads;
    const long step = (long)nq * gridDim.x * gridDim.y;
    for (long i = (long)(blockIdx.y * gridDim.x + blockIdx.x) * nq + (tid - kChainThreads); i < a.res.n4; i += step)
      reinterpret_cast<float4*>(a.res.dst)[i] = __ldcv(reinterpret_cast<const float4*>(a.res.src) + i);
  }
  if (!ok && (tid & 31) == 0) atomicOr(a.err, kErrTimeout);

  // ---- last CTA: top-k, softmax, routing ----
  if (a.ep_on) {
    // the barrier orders the CTA's peer stores before thread 0's system fence
    __syncthreads();
    if (tid == 0) __threadfence_system();
  } else {
    // the barrier orders the CTA's logit and activation stores before
    // thread 0's fence and arrival
    __syncthreads();
    if (tid == 0) __threadfence();
  }
  if (tid == 0) s_last = atomicAdd(a.counter, 1) == (int)(gridDim.x * gridDim.y) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  __shared__ int sidx[kMaxTK];
  __shared__ int cnt[kMaxE], start[kMaxE], s_tab[1 + 3 * kMaxTiles];
  __shared__ int s_route[2 + 2 * kMaxE + kMaxTK];
  const int lane = tid & 31, warp = tid >> 5;
  int TK = a.T * a.K;
  for (int i = tid; i < a.E_local; i += kThreads) cnt[i] = 0;
  // top-k per token: one warp per token, K rounds. Lane l holds the
  // contiguous experts l*PERL .. l*PERL+PERL-1, so lane order is expert order:
  // each round takes the largest order-preserving key of the warp (redux.sync)
  // and the lowest lane holding it (ballot), whose local pick is its lowest
  // expert with that key. Keys of NaN and -inf are 0 (never chosen) and -0 is
  // keyed as +0, so equal values tie exactly as in topk_desc's strict-'>'
  // insertion (lower index first). Lane r keeps round r's winner; the softmax
  // (:481-487) then runs across lanes, summing in order.
  // Each lane first sorts its PERL (key, expert) pairs, larger key first and
  // lower expert first on equal keys (a bitonic network on the 64-bit words
  // key << 32 | ~expert), so a round only compares the lanes' heads and the
  // winner shifts its list.
  constexpr int PERL = kMaxE / 32;
  static_assert(PERL == 8, "bitonic network of 8");
  for (int t = warp; t < a.T; t += kThreads / 32) {
    unsigned long long c[PERL];
#pragma unroll
    for (int i = 0; i < PERL; ++i) {
      const int e = lane * PERL + i;
      float v = e < a.E ? __ldcg(a.logits + (size_t)t * a.E + e) : -INFINITY;
      if (v == 0.0f) v = 0.0f;
      const unsigned u = __float_as_uint(v);
      const unsigned key = !(v > -INFINITY) ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
      c[i] = ((unsigned long long)key << 32) | (unsigned)~e;
    }
#pragma unroll
    for (int k = 2; k <= PERL; k <<= 1)
#pragma unroll
      for (int j = k >> 1; j > 0; j >>= 1)
#pragma unroll
        for (int i = 0; i < PERL; ++i) {
          const int l = i ^ j;
          if (l > i) {
            // descending where (i & k) == 0, ascending elsewhere: sorted descending at the end
            const bool sw = ((i & k) == 0) ? (c[i] < c[l]) : (c[i] > c[l]);
            const unsigned long long lo = sw ? c[l] : c[i], hi = sw ? c[i] : c[l];
            c[i] = lo; c[l] = hi;
          }
        }
    float myv = -INFINITY;
    int myi = -1;
    for (int r = 0; r < a.K; ++r) {
      const unsigned hk = (unsigned)(c[0] >> 32);
      const unsigned M = __reduce_max_sync(0xffffffffu, hk);
      if (M == 0u) break;                                        // only NaN / -inf left: no expert
      const int wl = __ffs(__ballot_sync(0xffffffffu, hk == M)) - 1;   // lowest lane = lowest expert
      const int I = (int)~__shfl_sync(0xffffffffu, (unsigned)c[0], wl);
      if (lane == r) {
        const unsigned u = (M & 0x80000000u) ? (M & 0x7fffffffu) : ~M;
        myv = __uint_as_float(u);
        myi = I;
      }
      if (lane == wl) {
#pragma unroll
        for (int i = 0; i < PERL - 1; ++i) c[i] = c[i + 1];
        c[PERL - 1] = 0ull;
      }
    }
    float mx = __shfl_sync(0xffffffffu, myv, 0);
    for (int i = 1; i < a.K; ++i) {
      const float vi = __shfl_sync(0xffffffffu, myv, i);
      if (vi > mx) mx = vi;
    }
    const float ev = lane < a.K ? exp_f32(__fsub_rn(myv, mx)) : 0.0f;
    float sum = 0.0f;
    for (int i = 0; i < a.K; ++i) sum = fadd(sum, __shfl_sync(0xffffffffu, ev, i));
    const float inv = fdiv(1.0f, fadd(sum, 1e-9f));
    if (lane < a.K) {
      const float pv = fmul(ev, inv);
      a.idx[t * a.K + lane] = myi;
      a.p[t * a.K + lane] = pv;
      sidx[t * a.K + lane] = myi;
      if (a.ep_on)
        for (int di = 0; di < a.ep.world; ++di) {
          uint8_t* pb = peer_base(a.ep, (a.ep.rank + 1 + di) % a.ep.world);
          const size_t s = (size_t)a.ep.rank * a.ep.T_local * a.K + t * a.K + lane;
          reinterpret_cast<int*>(pb + a.ep.idx_off)[s] = myi;
          reinterpret_cast<float*>(pb + a.ep.p_off)[s] = pv;
        }
    }
  }
  __syncthreads();
  if (a.ep_on) {
    // dispatch: raise this rank's flag at every rank, wait for every rank's,
    // then route the slots of all ranks' tokens (slot = global token * K + k)
    __shared__ int s_ok;
    if (tid == 0) {
      __threadfence_system();
      for (int di = 0; di < a.ep.world; ++di) {
        const int p = (a.ep.rank + 1 + di) % a.ep.world;
        st_release_sys(reinterpret_cast<unsigned long long*>(peer_base(a.ep, p) + kEpDispatchFlags) + a.ep.rank,
                       a.ep.seq);
      }
      s_ok = wait_flags_sys(reinterpret_cast<const unsigned long long*>(a.ep.base_local + kEpDispatchFlags),
                            a.ep.world, a.ep.seq, a.ep.wait_ns);
      if (!s_ok) atomicOr(a.err, kErrTimeout);
    }
    __syncthreads();
    // every rank's routing is done: if any rank marked a token out of range,
    // this rank's exact fix-up pass has slots to recompute (one peer per thread)
    if (s_ok && tid < a.ep.world &&
        *reinterpret_cast<volatile int*>(peer_base(a.ep, tid) + a.ep.xflag_off) == (int)a.ep.seq)
      a.flags[0] = 1;
    TK = s_ok ? a.ep.world * a.ep.T_local * a.K : 0;   // a failed wait routes nothing
    const int* all = reinterpret_cast<const int*>(a.ep.base_local + a.ep.idx_off);
    for (int s = tid; s < TK; s += kThreads) sidx[s] = __ldcg(all + s);
    __syncthreads();
  }
  for (int s = tid; s < TK; s += kThreads) {
    const int el = sidx[s] - a.e_begin;
    if (el >= 0 && el < a.E_local) atomicAdd(&cnt[el], 1);
  }
  if (a.hsum)
    for (int s = tid; s < TK; s += kThreads) a.hsum[s] = 0;
  __syncthreads();
  // exclusive scans over experts of (slots, active flag, tiles): one thread
  // per expert, warp shuffles, then the warp totals through shared memory
  static_assert(kMaxE <= kThreads, "one thread per expert");
  int* r_active = s_route + 1;
  int* r_off = s_route + 1 + a.E_local;
  const int mt = a.max_tiles;
  {
    __shared__ int s_wsum[3][kThreads / 32];
    const int el = tid;
    const int c = el < a.E_local ? cnt[el] : 0, act = c > 0;
    const int til = a.nt > 0 ? (c + a.nt - 1) / a.nt : 0;
    int xl = c, xa = act, xt = til;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int yl = __shfl_up_sync(0xffffffffu, xl, o), ya = __shfl_up_sync(0xffffffffu, xa, o),
                yt = __shfl_up_sync(0xffffffffu, xt, o);
      if (lane >= o) { xl += yl; xa += ya; xt += yt; }
    }
    if (lane == 31) { s_wsum[0][warp] = xl; s_wsum[1][warp] = xa; s_wsum[2][warp] = xt; }
    __syncthreads();
    for (int w = 0; w < warp; ++w) { xl += s_wsum[0][w]; xa += s_wsum[1][w]; xt += s_wsum[2][w]; }
    const int off = xl - c, na = xa - act, ntl = xt - til;      // exclusive prefixes
    if (el < a.E_local) {
      start[el] = off;
      if (c > 0) {
        r_active[na] = el;
        r_off[na] = off;
        for (int j0 = off, k = ntl; a.nt > 0 && j0 < off + c && k < mt; j0 += a.nt, ++k) {
          s_tab[1 + k] = na;
          s_tab[1 + mt + k] = j0;
          s_tab[1 + 2 * mt + k] = min(a.nt, off + c - j0);
        }
      }
      if (el == a.E_local - 1) {      // totals
        r_off[xa] = xl;
        s_route[0] = xa;
        s_tab[0] = xt < mt ? xt : mt;
      }
    }
    if (a.E_local == 0 && tid == 0) { r_off[0] = 0; s_route[0] = 0; s_tab[0] = 0; }
  }
  __syncthreads();
  // slot lists: placed with shared-memory atomics, then each expert's list is
  // sorted by slot id (one thread per expert) so the order is deterministic:
  // ascending slot within each expert, experts ascending
  int* r_slots = s_route + 2 + 2 * a.E_local;
  for (int i = tid; i < a.E_local; i += kThreads) cnt[i] = 0;
  __syncthreads();
  for (int s = tid; s < TK; s += kThreads) {
    const int el = sidx[s] - a.e_begin;
    if (el < 0 || el >= a.E_local) continue;
    r_slots[start[el] + atomicAdd(&cnt[el], 1)] = s;
  }
  __syncthreads();
  for (int el = tid; el < a.E_local; el += kThreads) {
    int* lst = r_slots + start[el];
    const int c = cnt[el];
    for (int i = 1; i < c; ++i) {
      const int v = lst[i];
      int j = i - 1;
      while (j >= 0 && lst[j] > v) { lst[j + 1] = lst[j]; --j; }
      lst[j + 1] = v;
    }
  }
  __syncthreads();
  if (a.slot_pos) {
    const int J = r_off[s_route[0]];
    for (int j = tid; j < J; j += kThreads) a.slot_pos[r_slots[j]] = j;
  }
  __syncthreads();
  // copy the tables out with all threads
  const int nr = 2 + 2 * a.E_local + TK;
  for (int i = tid; i < nr; i += kThreads) a.route[i] = s_route[i];
  if (a.nt > 0) {
    int* tab = a.route + nr;
    for (int i = tid; i < 1 + 3 * mt; i += kThreads) tab[i] = s_tab[i];
  }
  if (tid == 0) *a.counter = 0;
  MOE_TL_END(kTlRoute);
}

}  // namespace rt

bool decode_route_supported(const LayerDev& L, int T, const float* x) {
  const int El = L.e_end - L.e_begin;
  return T * L.topk <= rt::kMaxTK && L.E <= rt::kMaxE && El <= rt::kMaxE && L.topk <= 32 &&
         L.D % (16 * rt::kChunks) == 0 && (size_t)(rt::kE + rt::kT) * (L.D + 4) * 4 <= 200 * 1024 &&
         ((uintptr_t)x % 16) == 0 && ((uintptr_t)L.router_w % 16) == 0;
}

void launch_decode_route(const LayerDev& L, const Workspace& ws, const float* x, int T, int nt,
                         int* counter, int* err, cudaStream_t st, const EpView* ep, const RowCopy* res) {
  rt::Args a{};
  if (res) a.res = *res;
  a.x = x; a.W = L.router_w; a.b = L.router_b; a.T = T; a.E = L.E; a.D = L.D; a.K = L.topk;
  a.logits = ws.logits; a.idx = ws.topk_idx; a.p = ws.topk_p;
  a.route = ws.route; a.e_begin = L.e_begin; a.E_local = L.e_end - L.e_begin;
  a.hsum = L.dtype == 3 ? ws.hsum : nullptr;
  const int T_route = ep ? ep->world * ep->T_local : T;     // tokens whose slots are routed here
  a.nt = nt; a.max_tiles = nt > 0 ? route_max_tiles(T_route * L.topk, a.E_local, nt) : 0;
  a.slot_pos = nt > 0 ? ws.slot_pos : nullptr;
  a.xact = ws.xact; a.xsum = ws.xsum; a.q4_mma = nt > 0; a.counter = counter; a.err = err;
  a.flags = ws.xbad;
  a.ep_on = ep != nullptr;
  if (ep) a.ep = *ep;
  const size_t smem = (size_t)(rt::kE + rt::kT) * (L.D + 4) * 4;
  dim3 grid((L.E + rt::kE - 1) / rt::kE, (T + rt::kT - 1) / rt::kT);
  if (L.dtype == 2) {
    static size_t attr = 0;
    if (smem > attr) {
      cudaFuncSetAttribute(rt::decode_route_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attr = smem;
    }
    launch_pdl(rt::decode_route_kernel<8>, grid, dim3(rt::kThreads), smem, st, a);
  } else {
    static size_t attr = 0;
    if (smem > attr) {
      cudaFuncSetAttribute(rt::decode_route_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attr = smem;
    }
    launch_pdl(rt::decode_route_kernel<4>, grid, dim3(rt::kThreads), smem, st, a);
  }
}

MOE_TL_IO(router)

}  // namespace moe
