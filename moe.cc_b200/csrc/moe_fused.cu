// moe_fused.cu — decode expert FFN (Q8) as ONE persistent tcgen05 kernel:
// gate/up and down projections of all routed experts, with the dependency
// between them tracked per expert instead of per kernel.
//
// Units. A gate/up unit is (expert tile, 128-row block of F): 16 k-chunks of
// 128 bytes over D, gate and up weights. Its B operand is either the T token
// rows as they are (T <= NT: every expert has one tile of at most NT slots,
// the epilogue reads each slot's token column), or NT-slot tiles of the
// expert-sorted gathered rows (larger T: an expert may have several tiles).
// A down unit is (expert tile, 128-row block of D): 6 k-chunks over F, B =
// the tile's slot rows of h written by its gate/up units.
//
// Schedule. One global work counter hands out unit ids; ids [0, NG) are the
// gate/up units, [NG, NG+ND) the down units, so every gate/up unit is claimed
// before any down unit. A gate/up unit's epilogue warps each bump the
// expert's completion counter after storing their rows of h; the warp that
// completes it appends the expert to a ready list (release store). Down unit
// c takes 128-row block c % (D/128) of the (c / (D/128))-th expert to become
// ready, so the down units follow the order in which experts finish; its
// producer waits (bounded) only until that list entry is published. Gate/up
// units never wait and a unit is only claimed by a running CTA, so the waits
// cannot form a cycle.
// With the dependency per expert, the down weights of experts whose gate/up
// is done stream while other experts' gate/up still run: no kernel boundary,
// no drain and refill between the two projections.
//
// Shared memory: a ring of slots, each = one 128x128 weight tile (16 KB,
// 128B-swizzled, TMA) + one B pair (low / high activation limb, NT x 128 B
// each). A gate/up k-chunk takes two slots (gate tile + B, up tile); a down
// k-chunk one. TMEM: two accumulator buffers of 4*NT columns (gate lo/hi, up
// lo/hi; down uses the first 2*NT). Arithmetic is that of moe_mma.cu
// (kernels.c:51-93 Q8 dot products, exact int32, then the fp32 epilogues of
// test_model_trace.c:499-510), so results are bit-identical to it.
//
// Roles: warp 0 lane 0 = work claiming + TMA producer, warp 1 lane 0 = MMA
// issuer, warps 2..9 = epilogue (tcgen05.ld, one weight row per thread).
// Every wait is bounded (kWaitNs of %globaltimer): on expiry the CTA flags
// kErrTimeout and leaves, after waiting (bounded) for its own copies.
#include <cuda.h>
#include "common.cuh"
#include "kernels.cuh"
#include "pipeline.cuh"
#include "tc.cuh"
#include "tmap.cuh"

namespace moe {
namespace fz {
#ifdef MOE_TIMELINE
// per-CTA trace of the timeline build: [start, first claim, gate/up units,
// down units, ns stalled on expert dependencies, producer done, end]
__device__ unsigned long long g_fz_trace[512][8];
#define FZ_T(i, v) do { if (blockIdx.x < 512) g_fz_trace[blockIdx.x][i] = (v); } while (0)
#else
#define FZ_T(i, v) do { } while (0)
#endif

using mm::TMap;

constexpr int kUnitRing = 8;           // claimed unit ids published to the MMA / epilogue warps
constexpr int kA = 128 * 128;          // one weight tile (Q4: packed, two k-chunks)
constexpr int kAR = 2;                 // Q4: depth of the TMEM ring of expanded A tiles
// Q8: 8 epilogue warps. Q4: 4 epilogue + 8 nibble-expander warps (two CTAs
// per SM must fit the register file).
__host__ __device__ constexpr int epi_warps(int dt) { return dt == 4 ? 4 : 8; }
__host__ __device__ constexpr int exp_warps(int dt) { return dt == 4 ? 8 : 0; }
__host__ __device__ constexpr int threads(int dt) { return (2 + epi_warps(dt) + exp_warps(dt)) * 32; }

struct Args {
  const int* route; int E_local, TK, max_tiles, topk;
  const uint8_t* slab; size_t stride, gs_off, us_off, ds_off;
  int D, F;                            // hidden, intermediate
  uint8_t* hs0; uint8_t* hs1;          // h planes [J][F] (expert-sorted slots)
  float* ys;                           // [J][D] y rows (expert-sorted slots)
  int nslots, slot_bytes, w_once;
  int tokb;                            // 1: B of gate/up = the token rows (T <= NT); 0: the
                                       // expert-sorted gathered rows (tile j0...)
  int* ctr;                            // [0] work, [1] arrivals, [2] ready count, then per-tile
                                       // completion [kFusedMaxTiles] and the ready list [kFusedMaxTiles]
  int ep_on; EpView ep;
  const int* xsum; int* hsum;          // Q4 zero point: per-token Σa, per-slot Σh
  const int* xsum_s;                   // Q4, gathered rows: the token Σa of sorted slot j
  int* err;
  int* flags;                          // per-token range flags (range_fail) or null
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

template <int DT, int NT>
__global__ void __launch_bounds__(threads(DT), 2)
    moe_fused_kernel(const __grid_constant__ TMap tG, const __grid_constant__ TMap tU,
                     const __grid_constant__ TMap tX0, const __grid_constant__ TMap tX1,
                     const __grid_constant__ TMap tDn, const __grid_constant__ TMap tH0,
                     const __grid_constant__ TMap tH1, const Args a) {
  constexpr int B = NT * 128;                       // one activation tile (one limb, one k-chunk)
  constexpr bool Q4 = DT == 4;
  constexpr int KPS = Q4 ? 2 : 1;                   // k-chunks per slot (Q4: packed tile covers two)
  constexpr int NLB = Q4 ? 1 : 2;                   // activation limbs
  constexpr int ACC = 2 * NLB * NT;                 // accumulator columns per buffer (gate, up x limbs)
  constexpr int ACOL = 2 * ACC;                     // Q4: first TMEM column of the expanded-A ring
  constexpr int TNEED = 2 * ACC + (Q4 ? kAR * 2 * 32 : 0);
  constexpr uint32_t TCOLS = TNEED <= 128 ? 128 : 256;
  static_assert(TNEED <= 256, "two CTAs per SM share the 512 TMEM columns");
  constexpr float S = Q4 ? 7.0f : 127.0f;
  constexpr int kEpiWarps = epi_warps(DT), kExpWarp0 = 2 + kEpiWarps;
  MOE_TL_START(kTlGateup);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.nslots * a.slot_bytes);
  uint64_t* empty = full + a.nslots;
  __shared__ uint64_t acc_full[2], acc_empty[2], unit_rdy[kUnitRing], afull[kAR], aempty[kAR];
  __shared__ int s_unit[kUnitRing], s_utile[kUnitRing];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort, s_issued, s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    s_abort = 0; s_issued = 0;
    for (int s = 0; s < a.nslots; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], kEpiWarps); }
    for (int i = 0; i < kUnitRing; ++i) mbar_init(&unit_rdy[i], 1);
    if (Q4)
      for (int b = 0; b < kAR; ++b) { mbar_init(&afull[b], exp_warps(DT)); mbar_init(&aempty[b], 1); }
    fence_mbar_init();
    tc::prefetch_tmap(&tG.m); tc::prefetch_tmap(&tU.m); tc::prefetch_tmap(&tX0.m);
    tc::prefetch_tmap(&tX1.m); tc::prefetch_tmap(&tDn.m); tc::prefetch_tmap(&tH0.m);
    tc::prefetch_tmap(&tH1.m);
  }
  if (warp == 1) tc::tmem_alloc(&s_tmem, TCOLS);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = s_tmem;
  pdl_wait();          // the routing tables and token activations come from the kernels before
  pdl_launch();

  const TileView tv = tile_view(a.route, a.E_local, a.TK, a.max_tiles);
  const int* active = a.route + 1;
  const int* slots = a.route + 2 + 2 * a.E_local;
  const int nmg = a.F / 128, nmd = a.D / 128;
  const int kcg = a.D / 128, kcd = a.F / 128;        // k-chunks of a gate/up and of a down unit
  const int ntiles = *tv.n;
  const int NG = ntiles * nmg, NTOT = NG + ntiles * nmd;
  const int done_target = nmg * kEpiWarps;          // epilogue-warp signals per expert tile
  int* work = a.ctr;
  int* rcount = a.ctr + 2;
  int* done = a.ctr + 3;
  int* ready = a.ctr + 3 + kFusedMaxTiles;
  volatile int* abort_flag = &s_abort;

  if (warp == 0) {
    // ------------------- work claiming + TMA producer -------------------
    if (lane == 0) {
#ifdef MOE_TIMELINE
      unsigned long long n_gu = 0, n_dn = 0, stall = 0;
      FZ_T(0, tl_now());
#endif
      const uint64_t wpol = tc::policy_evict_first();
      // weight tile of slot stage ks: 128 bytes of every row (Q8: k-chunk ks;
      // Q4: packed k-chunks 2ks, 2ks+1)
      auto load_w = [&](const TMap& m, int ks, int mb, int e, uint8_t* dst, uint64_t* bar) {
        if (a.w_once) tc::tma_load_3d_hint(dst, &m.m, ks * 128, mb * 128, e, bar, wpol);
        else tc::tma_load_3d(dst, &m.m, ks * 128, mb * 128, e, bar);
      };
      // activations of stage ks into the slot's B region: Q8 both limbs of
      // k-chunk ks, Q4 the one limb of k-chunks 2ks and 2ks+1
      auto load_b = [&](const TMap& m0, const TMap& m1, int ks, int row, uint8_t* dst, uint64_t* bar) {
        if (Q4) {
          tc::tma_load_2d(dst, &m0.m, (2 * ks) * 128, row, bar);
          tc::tma_load_2d(dst + B, &m0.m, (2 * ks + 1) * 128, row, bar);
        } else {
          tc::tma_load_2d(dst, &m0.m, ks * 128, row, bar);
          tc::tma_load_2d(dst + B, &m1.m, ks * 128, row, bar);
        }
      };
      int it = 0, ul = 0;                    // slot items issued, units claimed
      int nxt = atomicAdd(work, 1);
      for (;; ++ul) {
        const int g = nxt;
        const int ri = ul % kUnitRing;
        bool stop = g >= NTOT || *abort_flag;
        int tile = 0;
        if (!stop && g >= NG) {
          // down unit: its expert is the ((g - NG) / (D/128))-th to finish gate/up
          const int pos = (g - NG) / nmd;
          uint32_t i = 0;
#ifdef MOE_TIMELINE
          const unsigned long long w0 = tl_now();
#endif
          int v;
          const uint64_t t0 = globaltimer_ns();   // bounded by time (kWaitNs), checked every 64 polls
          while ((v = ld_acquire_gpu(ready + pos)) == 0)
            if ((++i & 63) == 0 && globaltimer_ns() - t0 > kWaitNs) break;
#ifdef MOE_TIMELINE
          stall += tl_now() - w0;
#endif
          if (v == 0) { atomicOr(a.err, kErrTimeout); *abort_flag = 1; stop = true; }
          tile = v - 1;
          fence_proxy_async_global();        // generic stores of h -> the tensor copies below
        }
        s_unit[ri] = stop ? -1 : g;
        s_utile[ri] = tile;
        mbar_arrive(&unit_rdy[ri]);          // release: the id is visible to the consumers
        if (stop) break;
#ifdef MOE_TIMELINE
        if (ul == 0) FZ_T(1, tl_now());
        if (g < NG) ++n_gu; else ++n_dn;
#endif
        nxt = atomicAdd(work, 1);            // next claim in flight while this unit streams
        // one slot item: wait the slot free, expect its bytes
        auto take = [&](uint32_t bytes) -> int {
          const int st = it % a.nslots;
          if (it >= a.nslots && !mbar_wait(&empty[st], ((it / a.nslots) - 1) & 1, kWaitNs)) {
            atomicOr(a.err, kErrTimeout); *abort_flag = 1; return -1;
          }
          mbar_arrive_expect_tx(&full[st], bytes);
          ++it;
          s_issued = it;
          return st;
        };
        if (g < NG) {
          const int tile = g / nmg, mb = g % nmg, e = active[tv.u[tile]];
          const int by = a.tokb ? 0 : tv.j0[tile];   // token rows, or this tile's gathered rows
          for (int ks = 0; ks < kcg / KPS && !*abort_flag; ++ks) {
            const int s0 = take(kA + 2 * B);
            if (s0 < 0) break;
            uint8_t* p0 = smem + (size_t)s0 * a.slot_bytes;
            load_w(tG, ks, mb, e, p0, &full[s0]);
            load_b(tX0, tX1, ks, by, p0 + kA, &full[s0]);
            const int s1 = take(kA);
            if (s1 < 0) break;
            load_w(tU, ks, mb, e, smem + (size_t)s1 * a.slot_bytes, &full[s1]);
          }
        } else {
          const int mb = (g - NG) % nmd, e = active[tv.u[tile]], j0 = tv.j0[tile];
          for (int ks = 0; ks < kcd / KPS && !*abort_flag; ++ks) {
            const int s0 = take(kA + 2 * B);
            if (s0 < 0) break;
            uint8_t* p0 = smem + (size_t)s0 * a.slot_bytes;
            load_w(tDn, ks, mb, e, p0, &full[s0]);
            load_b(tH0, tH1, ks, j0, p0 + kA, &full[s0]);
          }
        }
      }
#ifdef MOE_TIMELINE
      FZ_T(2, n_gu); FZ_T(3, n_dn); FZ_T(4, stall); FZ_T(5, tl_now());
#endif
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      // Q8: A = s8 weights (shared memory), B = u8 low limb / s8 high limb.
      // Q4: A = u8 nibbles (expanded into tensor memory), B = s8 activations.
      const uint32_t idesc_lo = tc::idesc_i8(128, NT, !Q4, Q4);
      const uint32_t idesc_hi = tc::idesc_i8(128, NT, true, true);
      int it = 0, ik = 0;                     // slot items consumed, Q4 expanded k-chunks consumed
      for (int ul = 0;; ++ul) {
        const int ri = ul % kUnitRing;
        if (!mbar_wait(&unit_rdy[ri], (ul / kUnitRing) & 1, kWaitNs)) {
          atomicOr(a.err, kErrTimeout); *abort_flag = 1; break;
        }
        const int g = s_unit[ri];
        if (g < 0) break;
        const int buf = ul & 1;
        if (ul >= 2 && !mbar_wait(&acc_empty[buf], ((ul >> 1) - 1) & 1, kWaitNs)) {
          atomicOr(a.err, kErrTimeout); *abort_flag = 1; break;
        }
        tc::fence_after_sync();
        const uint32_t dbase = tmem + buf * ACC;
        const bool gu = g < NG;
        const int nst = (gu ? kcg : kcd) / KPS;
        bool bad = false;
        for (int ks = 0; ks < nst && !bad; ++ks) {
          const int s0 = it % a.nslots, ph0 = (it / a.nslots) & 1;
          ++it;
          int s1 = -1, ph1 = 0;
          if (gu) { s1 = it % a.nslots; ph1 = (it / a.nslots) & 1; ++it; }
          const uint8_t* p0 = smem + (size_t)s0 * a.slot_bytes;
          if (!Q4) {
            if (!mbar_wait(&full[s0], ph0, kWaitNs) || (gu && !mbar_wait(&full[s1], ph1, kWaitNs))) {
              bad = true; break;
            }
            tc::fence_after_sync();
            const uint64_t db0 = tc::sw128_desc(p0 + kA), db1 = tc::sw128_desc(p0 + kA + B);
            const uint64_t da0 = tc::sw128_desc(p0);
            const uint64_t da1 = gu ? tc::sw128_desc(smem + (size_t)s1 * a.slot_bytes) : 0;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t acc = (ks | kk) != 0;
              tc::mma_i8(dbase + 0 * NT, da0 + 2 * kk, db0 + 2 * kk, idesc_lo, acc);
              tc::mma_i8(dbase + 1 * NT, da0 + 2 * kk, db1 + 2 * kk, idesc_hi, acc);
              if (gu) {
                tc::mma_i8(dbase + 2 * NT, da1 + 2 * kk, db0 + 2 * kk, idesc_lo, acc);
                tc::mma_i8(dbase + 3 * NT, da1 + 2 * kk, db1 + 2 * kk, idesc_hi, acc);
              }
            }
          } else {
            // the expanders saw the slots full before releasing each k-chunk
            for (int q = 0; q < KPS; ++q, ++ik) {
              const int ab = ik % kAR;
              if (!mbar_wait(&afull[ab], (ik / kAR) & 1, kWaitNs)) { bad = true; break; }
              tc::fence_after_sync();
              const uint64_t db = tc::sw128_desc(p0 + kA + q * B);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint32_t acc = (ks | q | kk) != 0;
                // A: 32 TMEM columns per tile (gate / down at ring slot ab*2, up at ab*2+1)
                tc::mma_i8_ts(dbase, tmem + ACOL + (ab * 2) * 32 + kk * 8, db + 2 * kk, idesc_lo, acc);
                if (gu) tc::mma_i8_ts(dbase + NT, tmem + ACOL + (ab * 2 + 1) * 32 + kk * 8, db + 2 * kk, idesc_lo, acc);
              }
              tc::mma_commit(&aempty[ab]);
            }
            if (bad) break;
          }
          tc::mma_commit(&empty[s0]);
          if (gu) tc::mma_commit(&empty[s1]);
        }
        if (bad) { atomicOr(a.err, kErrTimeout); *abort_flag = 1; break; }
        tc::mma_commit(&acc_full[buf]);
      }
    }
  } else if (Q4 && warp >= kExpWarp0) {
    // --------------------- Q4 nibble expanders -> TMEM ----------------------
    // Warp = (TMEM lane quarter, part): gate/up units: part 0 unpacks the gate
    // tile, part 1 the up tile; down units: part p unpacks columns 16p..16p+15.
    // Row r's 64 packed bytes of k-chunk q (128B-swizzled: chunk h of the row
    // at h ^ (r & 7)) become 128 bytes = 32 TMEM columns: packed chunk c ->
    // columns 8c..8c+3 (its low nibbles) and 8c+4..8c+7 (its high nibbles),
    // the k order of the activations (q4_mma_pos).
    const int quarter = warp & 3, part = (warp - kExpWarp0) >> 2, r = quarter * 32 + lane;
    auto unpack = [&](const uint8_t* prow, int q, int c, uint32_t* o) {
      const uint4 w = *reinterpret_cast<const uint4*>(prow + ((((q << 2) + c) ^ (r & 7)) << 4));
      o[0] = w.x & 0x0F0F0F0Fu; o[1] = w.y & 0x0F0F0F0Fu; o[2] = w.z & 0x0F0F0F0Fu; o[3] = w.w & 0x0F0F0F0Fu;
      o[4] = (w.x >> 4) & 0x0F0F0F0Fu; o[5] = (w.y >> 4) & 0x0F0F0F0Fu;
      o[6] = (w.z >> 4) & 0x0F0F0F0Fu; o[7] = (w.w >> 4) & 0x0F0F0F0Fu;
    };
    int it = 0, ik = 0;
    for (int ul = 0;; ++ul) {
      const int ri = ul % kUnitRing;
      if (!mbar_wait(&unit_rdy[ri], (ul / kUnitRing) & 1, kWaitNs)) {
        if (lane == 0) { atomicOr(a.err, kErrTimeout); *abort_flag = 1; }
        break;
      }
      const int g = s_unit[ri];
      if (g < 0) break;
      const bool gu = g < NG;
      const int nst = (gu ? kcg : kcd) / KPS;
      bool bad = false;
      for (int ks = 0; ks < nst && !bad; ++ks) {
        int sm = it % a.nslots, ph = (it / a.nslots) & 1;
        ++it;
        if (gu) {
          if (part == 1) { sm = it % a.nslots; ph = (it / a.nslots) & 1; }
          ++it;
        }
        if (!mbar_wait(&full[sm], ph, kWaitNs)) { bad = true; break; }
        const uint8_t* prow = smem + (size_t)sm * a.slot_bytes + r * 128;
        for (int q = 0; q < KPS; ++q, ++ik) {
          const int ab = ik % kAR;
          if (ik >= kAR && !mbar_wait(&aempty[ab], ((ik / kAR) - 1) & 1, kWaitNs)) { bad = true; break; }
          const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + ACOL + (ab * 2) * 32;
          if (gu) {
            uint32_t o[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) unpack(prow, q, c, o + 8 * c);
            tc::tmem_st32(trow + part * 32, o);
          } else {
            uint32_t o[16];
#pragma unroll
            for (int c = 0; c < 2; ++c) unpack(prow, q, 2 * part + c, o + 8 * c);
            tc::tmem_st16(trow + 16 * part, o);
          }
          tc::tmem_wait_st();
          tc::fence_before_sync();            // TMEM stores -> the MMA thread after the barrier
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[ab]);
        }
      }
      if (bad) {
        if (lane == 0) { atomicOr(a.err, kErrTimeout); *abort_flag = 1; }
        break;
      }
    }
  } else {
    // ------------------------------- epilogue -------------------------------
    const int q = warp & 3, half = (warp - 2) >> 2, r = q * 32 + lane;
    for (int ul = 0;; ++ul) {
      const int ri = ul % kUnitRing;
      if (!mbar_wait(&unit_rdy[ri], (ul / kUnitRing) & 1, kWaitNs)) {
        if (lane == 0) { atomicOr(a.err, kErrTimeout); *abort_flag = 1; }
        break;
      }
      const int g = s_unit[ri], dtile = s_utile[ri];
      if (g < 0) break;
      const int buf = ul & 1;
      if (!mbar_wait(&acc_full[buf], (ul >> 1) & 1, kWaitNs)) {
        if (lane == 0) { atomicOr(a.err, kErrTimeout); *abort_flag = 1; }
        break;
      }
      tc::fence_after_sync();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * ACC;
      if (g < NG) {
        const int tile = g / nmg, mb = g % nmg, e = active[tv.u[tile]];
        const int j0 = tv.j0[tile], nt = tv.cnt[tile], n = mb * 128 + r;
        const uint8_t* ex = a.slab + (size_t)e * a.stride;
        const float sg = __ldg(reinterpret_cast<const float*>(ex + a.gs_off) + n);
        const float su = __ldg(reinterpret_cast<const float*>(ex + a.us_off) + n);
        // token rows: accumulator column t is token t, each routed slot reads its
        // token's column; gathered rows: column jj is the tile's slot jj
        for (int jj = half; jj < nt; jj += kEpiWarps / 4) {
          const int j = j0 + jj;
          const int t = a.tokb ? __ldg(slots + j) / a.topk : jj;      // warp-uniform column
          constexpr int NX = 2 * NLB;                                   // gate, up x limbs
          uint32_t v[NX][8], raw[NX];
#pragma unroll
          for (int x = 0; x < NX; ++x) tc::tmem_ld8(tbase + x * NT + (t & ~7), v[x]);
          tc::tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < NX; ++x) {
            raw[x] = v[x][0];
#pragma unroll
            for (int c = 1; c < 8; ++c) if ((t & 7) == c) raw[x] = v[x][c];
          }
          int dg, du;
          if (Q4) {   // nibbles are stored +8: subtract 8 * Σ activation of the token (exact mod 2^32)
            const unsigned as = 8u * (unsigned)(a.tokb ? __ldg(a.xsum + __ldg(slots + j) / a.topk)
                                                       : __ldg(a.xsum_s + j));
            dg = (int)(raw[0] - as);
            du = (int)(raw[1] - as);
          } else {
            dg = (int)(raw[0] + (raw[1] << 8));
            du = (int)(raw[2] + (raw[3] << 8));
          }
          const float gv = fmul(div_qscale(dg, !Q4), sg);
          const float uv = fmul(div_qscale(du, !Q4), su);
          const int ha = trunc_scale(fmul(silu_ref(gv), uv), S);
          if (Q4) {
            if (ha < -128 || ha > 127) range_fail(a.err, a.flags, __ldg(slots + j) / a.topk);
            a.hs0[(size_t)j * a.F + q4_mma_pos(n)] = (uint8_t)(ha & 0xFF);
            // Σ h of slot j for the down projection's zero-point correction
            const int hw = __reduce_add_sync(0xffffffffu, ha);
            if (lane == 0) atomicAdd(a.hsum + j, hw);
          } else {
            if (ha < -32768 || ha > 32767) range_fail(a.err, a.flags, __ldg(slots + j) / a.topk);
            a.hs0[(size_t)j * a.F + n] = (uint8_t)(ha & 0xFF);
            a.hs1[(size_t)j * a.F + n] = (uint8_t)((ha >> 8) & 0xFF);
          }
        }
        // this warp's rows of h are stored: count it toward the expert's completion
        __threadfence();
        __syncwarp();
        if (lane == 0 && atomicAdd(done + tile, 1) == done_target - 1) {
          // the expert's h is complete: publish it on the ready list
          const int pos = atomicAdd(rcount, 1);
          st_release_gpu(ready + pos, tile + 1);
        }
      } else {
        const int tile = dtile, mb = (g - NG) % nmd, e = active[tv.u[tile]];
        const int j0 = tv.j0[tile], nt = tv.cnt[tile], n = mb * 128 + r;
        const uint8_t* ex = a.slab + (size_t)e * a.stride;
        const float sd = __ldg(reinterpret_cast<const float*>(ex + a.ds_off) + n);
        for (int c0 = 8 * half; c0 < nt; c0 += 8 * (kEpiWarps / 4)) {
          uint32_t v0[8], v1[8];
          tc::tmem_ld8(tbase + c0, v0);
          if (!Q4) tc::tmem_ld8(tbase + NT + c0, v1);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (c0 + i >= nt) break;
            const int j = j0 + c0 + i;
            // Q4: the down nibbles are stored +8: subtract 8 * Σ h of the slot
            // (complete: all the tile's gate/up units finished before this claim)
            const int dot = Q4 ? (int)(v0[i] - 8u * (unsigned)__ldcg(a.hsum + j)) : (int)(v0[i] + (v1[i] << 8));
            const float yv = fmul(div_qscale(dot, !Q4), sd);
            if (a.ep_on) {
              const int sl = __ldg(slots + j), per = a.topk * a.ep.T_local, owner = sl / per;
              float* yo = reinterpret_cast<float*>(
                  __ldg(reinterpret_cast<const unsigned long long*>(a.ep.base) + owner) + a.ep.y_off);
              yo[(size_t)(sl - owner * per) * a.D + n] = yv;
            } else {
              a.ys[(size_t)j * a.D + n] = yv;
            }
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && s_abort) {
    // let the tensor copies still in flight land before the CTA's smem goes away
    for (int i = max(0, s_issued - a.nslots); i < s_issued; ++i)
      mbar_wait(&full[i % a.nslots], (i / a.nslots) & 1, kWaitNs);
  }
  // The last CTA out resets the work and completion counters for the next
  // call and, expert-parallel, raises this rank's combine flag at every rank,
  // unless a token was marked out of range (by any rank's routing, or by an
  // epilogue here): then the exact fix-up pass that follows raises them.
  if (threadIdx.x == 0) {
    if (a.ep_on) __threadfence_system(); else __threadfence();
    s_last = atomicAdd(a.ctr + 1, 1) == (int)gridDim.x - 1;
    if (s_last) {
      __threadfence();
      a.ctr[0] = 0;
      a.ctr[1] = 0;
      a.ctr[2] = 0;
      for (int i = 0; i < ntiles; ++i) { done[i] = 0; ready[i] = 0; }
      if (a.ep_on && !(a.flags && *reinterpret_cast<volatile int*>(a.flags)))
        ep_raise_combine(a.ep);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TCOLS);
  }
  MOE_TL_END(kTlGateup);
#ifdef MOE_TIMELINE
  if (threadIdx.x == 0) FZ_T(6, tl_now());
#endif
}

}  // namespace fz

#ifdef MOE_TIMELINE
void fz_trace_read(unsigned long long* out) { cudaMemcpyFromSymbol(out, fz::g_fz_trace, sizeof(fz::g_fz_trace)); }
#endif

// Q8 only. Up to 32 tokens the gate/up B operand is the token rows (every
// expert's slots fit one tile); above, 32-slot tiles of the expert-sorted
// gathered rows (an expert with more slots has several tiles, each with its
// own completion count). Used from 8 tokens up: below that there are fewer
// gate/up units than CTAs, every expert completes at the same late moment and
// the down claims only wait (measured, Qwen3-30B-A3B layer: T=1 50.1 vs 43.2
// us two-kernel, T=4 57.7 vs 54.8; T=8 75.6 vs 77.5, T=16 94.7 vs 96.0, T=24
// 108.7 vs 118.7, T=32 115.9 vs 125.7). MOE_FUSED=0 never uses it, 2 for
// every decode size; MOE_FUSED_MAX_T bounds the gathered sizes.
int fused_tile_n(const LayerDev& L, int T) {
  static int env = -1, tmax = -1;
  if (env < 0) { const char* e = getenv("MOE_FUSED"); env = e ? atoi(e) : 1; }
  if (tmax < 0) { const char* e = getenv("MOE_FUSED_MAX_T"); tmax = e ? atoi(e) : 256; }
  const int kq = L.dtype == 3 ? 256 : 128;   // Q4: two k-chunks per stage
  if (!env || (T < 8 && env != 2) || T > tmax || (L.dtype != 2 && L.dtype != 3) || L.D % kq || L.F % kq) return 0;
  const int nt = T <= 16 ? 16 : 32;
  if (route_max_tiles(T * L.topk, L.e_end - L.e_begin, nt) > kFusedMaxTiles) return 0;
  return nt;
}

bool launch_mma_fused(const LayerDev& L, const Workspace& ws, int T, int nt, int* err, cudaStream_t st,
                      const EpView* ep) {
  using namespace mm;
  const int E_local = L.e_end - L.e_begin, TK = T * L.topk, cap = ws.cap_T * ws.cap_K;
  const bool tokb = T <= nt, q4 = L.dtype == 3;
  TMap tG, tU, tX0, tX1, tDn, tH0, tH1;
  // activations: token rows (2*D pitch) or the gathered planes; Q4 has one limb
  // (plane 0), so the second map repeats the first
  const bool xmap = tokb ? (map_rows(tX0, ws.xact, L.D, ws.cap_T, nt, 2 * L.D) &&
                            map_rows(tX1, q4 ? ws.xact : ws.xact + L.D, L.D, ws.cap_T, nt, 2 * L.D))
                         : (map_rows(tX0, ws.xs0, L.D, cap, nt) && map_rows(tX1, q4 ? ws.xs0 : ws.xs1, L.D, cap, nt));
  if (!xmap || !map_weights(tG, L, L.gq_off, L.D, L.F) || !map_weights(tU, L, L.uq_off, L.D, L.F) ||
      !map_weights(tDn, L, L.dq_off, L.F, L.D) || !map_rows(tH0, ws.hs0, L.F, cap, nt) ||
      !map_rows(tH1, q4 ? ws.hs0 : ws.hs1, L.F, cap, nt))
    return false;
  fz::Args a{};
  a.route = ws.route; a.E_local = E_local; a.TK = TK; a.max_tiles = route_max_tiles(TK, E_local, nt);
  a.topk = L.topk;
  a.slab = L.slab; a.stride = L.expert_stride; a.gs_off = L.gs_off; a.us_off = L.us_off; a.ds_off = L.ds_off;
  a.D = L.D; a.F = L.F; a.hs0 = ws.hs0; a.hs1 = ws.hs1; a.ys = ws.y;
  a.w_once = tokb && evict_first_on() ? 1 : 0;   // gathered: an expert may have several tiles
  a.tokb = tokb ? 1 : 0;
  a.ctr = ws.fused_ctr; a.err = err; a.flags = ws.xbad;
  a.xsum = ws.xsum; a.hsum = ws.hsum; a.xsum_s = ws.xsum_s;
  a.ep_on = ep != nullptr;
  if (ep) a.ep = *ep;
  a.slot_bytes = fz::kA + 2 * nt * 128;
  const int budget = 220 * 1024 / 2;
  a.nslots = (budget - 1024 - 256) / a.slot_bytes;
  if (a.nslots > 8) a.nslots = 8;
  if (a.nslots < 2) return false;
  const size_t smem = (size_t)a.nslots * a.slot_bytes + 1024 + 16 * (size_t)a.nslots;
  const int grid = 2 * sms();
  auto run = [&](auto kern, int idx, int nthreads) -> bool {
    static size_t attr[4] = {0, 0, 0, 0};
    size_t& at = attr[idx];
    if (smem > at) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return false;
      at = smem;
    }
    return launch_pdl(kern, dim3(grid), dim3(nthreads), smem, st, tG, tU, tX0, tX1, tDn, tH0, tH1, a) ==
           cudaSuccess;
  };
  if (q4) return nt == 16 ? run(fz::moe_fused_kernel<4, 16>, 2, fz::threads(4))
                          : run(fz::moe_fused_kernel<4, 32>, 3, fz::threads(4));
  return nt == 16 ? run(fz::moe_fused_kernel<8, 16>, 0, fz::threads(8)) : run(fz::moe_fused_kernel<8, 32>, 1, fz::threads(8));
}

MOE_TL_IO(moe_fused)

}  // namespace moe
