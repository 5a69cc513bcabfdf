// moe_mma.cu — routed-expert GEMMs on the 5th-generation tensor cores.
//
// D[128 weight rows][NT routed slots] = W_tile[128 x K] · X[NT x K]^T with
// tcgen05.mma kind::i8 (exact int32 accumulation in TMEM). Weights are the A
// operand (one 128-row block of one expert per tile, TMA 3-D tensor map over
// the per-expert slabs, 128-byte swizzle); the routed tokens' truncated
// activations, sorted by expert into contiguous rows, are the B operand
// (TMA 2-D). Q8 activations need 16 bits, so they are two byte limbs (lo as
// u8, hi as s8) and two MMAs; the epilogue recombines lo + 256*hi.
//
// Warp roles (persistent CTA, one per SM):
//   warp 0      TMA producer (one elected thread), S-stage smem ring
//   warp 1      TMEM allocator + MMA issuer (one elected thread)
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, one weight row per
//               thread, every (row, slot) finished in parallel:
//                 GATEUP: h = silu(g)*u, re-truncated for the down projection
//                         (test_model_trace.c:496-501, kernels.c:66/:113)
//                 DOWN:   y = dot/S*s (:502-503), rows for the separate
//                         k-ordered combine (:513-517)
// TMEM holds two accumulator buffers so the MMAs of tile i+1 overlap the
// epilogue of tile i. Every wait is bounded (kWaitNs of %globaltimer); on expiry the
// kernel flags kErrTimeout and leaves instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"
#include "tmap.cuh"

#include <stdlib.h>

namespace moe {
namespace mm {
#ifdef MOE_TIMELINE
// timeline build: per-stage clock64 stamps of CTA 0 of the Q4 gate/up kernel
// [stage][producer issued, expander saw data, expander done, MMA issued]
__device__ long long g_q4_trace[64][4];
#define Q4T(i, k) do { if (DT == 4 && MODE == GATEUP && blockIdx.x == 0 && (i) < 64) g_q4_trace[i][k] = clock64(); } while (0)
#else
#define Q4T(i, k) do { } while (0)
#endif

enum { GATEUP = 0, DOWN = 1 };
// Epilogue warps: several per TMEM lane quarter, splitting the slot columns.
// Wide (prefill) tiles need 16 to hide the epilogue's latency; decode tiles
// (<= 32 slots) use 8, which keeps two CTAs resident per SM.
// Q4 decode tiles keep the expanded weights in tensor memory (the MMA reads A
// from TMEM): the expanders unpack each thread's packed row in registers and
// store it with tcgen05.st, so neither the expanded tile's write nor the
// MMA's read goes through shared memory (in shared memory the expansion made
// the decode pipeline shared-memory-bandwidth bound).
#ifndef MOE_Q4_TMEM
#define MOE_Q4_TMEM 1
#endif
__host__ __device__ constexpr bool q4_a_in_tmem(int dt, int nt) { return MOE_Q4_TMEM && dt == 4 && nt <= 32; }
// Epilogue warps: 16 for wide tiles, 8 for decode tiles, 4 for Q4 decode
// (whose two CTAs per SM need the registers; decode tiles have few slots).
__host__ __device__ constexpr int epi_warps(int nt, int dt = 8) {
  return nt >= 64 ? 16 : (dt == 4 && MOE_Q4_TMEM) ? 4 : 8;
}
// Q4 nibble-expander warps: the expansion paces the decode pipeline, so small
// tiles get 8 (the wide prefill tiles keep 4 and their threads for the epilogue)
#ifndef MOE_Q4_EXP_DECODE
#define MOE_Q4_EXP_DECODE 8
#endif
__host__ __device__ constexpr int exp_warps(int dt, int nt) { return dt == 4 ? (nt <= 32 ? MOE_Q4_EXP_DECODE : 4) : 0; }
__host__ __device__ constexpr int cta_threads(int dt, int nt) { return (2 + epi_warps(nt, dt) + exp_warps(dt, nt)) * 32; }
// Q4 weights are loaded as 128-byte-wide, 128B-swizzled boxes: two k-chunks
// (256 nibbles) per row and per pipeline stage, so one tensor copy per matrix
// feeds two expansions and the swizzle spreads the expanders' row reads over
// all shared-memory banks.
constexpr int kQ4KPerStage = 2;
// Depth of the Q4 expanded-tile ring: the expanders run this many k-chunks
// ahead of the MMAs (2 and 4 measured the same for decode; the wide prefill
// tiles need the shared memory for their B operands).
#ifndef MOE_Q4_ARING
#define MOE_Q4_ARING 2
#endif
__host__ __device__ constexpr int q4_aring_depth(int nt) { return nt <= 32 ? MOE_Q4_ARING : 2; }



struct Args {
  int rows;          // output rows per expert (F for GATEUP, D for DOWN)
  int kchunks;       // K bytes / 128
  int n_mblk;        // rows / 128
  int stages, stage_bytes;
  const int* route;  // routing lists + tile table (route_view / tile_view)
  int E_local, TK, max_tiles;
  const uint8_t* slab;
  size_t stride, s0_off, s1_off;
  int F;                                   // GATEUP: output plane row length
  uint8_t* hs0; uint8_t* hs1;              // GATEUP outputs (expert-sorted rows)
  float* ys;                               // DOWN output [J][D]
  int T, topk;
  const int* xsum; int* hsum;                // Q4 zero-point sums (token / slot)
  const int* xsum_s;                         // Q4, gathered B rows: the token sum of sorted slot j
  int tokb;                                  // GATEUP: B = all T token rows (decode, T <= NT)
  int w_once;                                // T <= NT: one token tile per expert, weights read once
  int ep_on; EpView ep;                      // DOWN, expert parallel: slot rows go to their owners' y buffers
  int* err;
  int* flags;                                // per-token range flags (range_fail) or null
};

template <int DT, int MODE, int NT>
__global__ void __launch_bounds__(cta_threads(DT, NT), (DT == 4 && MOE_Q4_TMEM && NT <= 32) ? 2 : 1)
    moe_mma_kernel(const __grid_constant__ TMap tmA0, const __grid_constant__ TMap tmA1,
                   const __grid_constant__ TMap tmB0, const __grid_constant__ TMap tmB1, const Args a) {
  constexpr int kEpiWarps = epi_warps(NT, DT), kEpiPerQ = kEpiWarps / 4, kExpWarp0 = 2 + kEpiWarps;
  constexpr int kExpWarps = exp_warps(DT, NT), kExpThreads = kExpWarps * 32;
  constexpr int NM = MODE == GATEUP ? 2 : 1;     // weight matrices per tile
  constexpr int NL = DT == 8 ? 2 : 1;            // activation limbs
  constexpr int ACC = NM * NL * NT;              // accumulator columns per buffer
  constexpr bool ATM = q4_a_in_tmem(DT, NT);
  constexpr int ACOL = 2 * ACC;                  // ATM: first TMEM column of the expanded-A ring
  constexpr int TNEED = 2 * ACC + (ATM ? q4_aring_depth(NT) * NM * 32 : 0);
  constexpr uint32_t TCOLS = TNEED <= 32 ? 32 : TNEED <= 64 ? 64 : TNEED <= 128 ? 128
                             : TNEED <= 256 ? 256 : 512;
  static_assert(TNEED <= 512, "accumulators exceed TMEM");
  static_assert(!ATM || exp_warps(DT, NT) == 8, "TMEM expansion: one warp per (lane quarter, matrix or half)");
  constexpr float S = DT == 8 ? 127.0f : 7.0f;
  constexpr int A_BYTES = 128 * 128;              // one weight tile (Q4: two packed k-chunks)
  constexpr int B_BYTES = NT * 128;               // one activation limb tile of one k-chunk
  constexpr int KPS = DT == 4 ? kQ4KPerStage : 1;  // k-chunks per pipeline stage

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.stages * a.stage_bytes);
  uint64_t* empty = full + a.stages;
  uint64_t* acc_full = empty + a.stages;     // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  constexpr int AR = q4_aring_depth(NT);
  uint64_t* afull = acc_empty + 2;           // [AR] Q4: expanded A tiles written
  uint64_t* aempty = afull + AR;             // [AR] Q4: expanded A tiles consumed by the MMAs
  // Q4: the stage ring holds [packed tiles | B]; the expanded A tiles live in
  // their own AR-deep ring after the barriers (1024-aligned)
  uint8_t* aring = smem + (((size_t)a.stages * a.stage_bytes + 16 * (size_t)a.stages + 32 + 16 * AR + 1023) &
                           ~(size_t)1023);
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort, s_issued;

  MOE_TL_START(MODE == GATEUP ? kTlGateup : kTlDown);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const TileView tv = tile_view(a.route, a.E_local, a.TK, a.max_tiles);
  const int* active = a.route + 1;

  if (threadIdx.x == 0) {
    s_abort = 0; s_issued = 0;
    for (int s = 0; s < a.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], kEpiWarps); }
    if (DT == 4)
      for (int b = 0; b < AR; ++b) { mbar_init(&afull[b], kExpWarps); mbar_init(&aempty[b], 1); }
    fence_mbar_init();
    tc::prefetch_tmap(&tmA0.m); tc::prefetch_tmap(&tmB0.m);
    if (NM == 2) tc::prefetch_tmap(&tmA1.m);
    if (NL == 2) tc::prefetch_tmap(&tmB1.m);
  }
  if (warp == 1) tc::tmem_alloc(&s_tmem, TCOLS);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = s_tmem;
  // Dependent launch: gate/up reads the routing tables of the kernel right
  // before it, so it waits here. The down projection needs the gate/up output
  // only for its B operand: its routing tables are two launches old (complete),
  // so its producer first streams the weights of the first stages and waits
  // only before the first B load; the other warps wait here.
  if (MODE == GATEUP || threadIdx.x != 0) { pdl_wait(); pdl_launch(); }

  // units are dealt round-robin: tiles of heavily loaded experts (full slot
  // columns, the costliest epilogues) sit next to each other in the tile table
  const int n_units = *tv.n * a.n_mblk;
  const int u0 = blockIdx.x, ustep = gridDim.x;
  volatile int* abort_flag = &s_abort;

  if (warp == 0) {
    // ------------------------- TMA producer -------------------------
    if (lane == 0) {
      const uint32_t bytes = NM * A_BYTES + KPS * NL * B_BYTES;
      const uint64_t wpol = tc::policy_evict_first();
      // f(unit, kc, it) over this CTA's k-chunk iterations, until it returns
      // false; the unit's expert, row block and first slot are read once
      struct Unit { int e, mb, j0; };
      auto for_iters = [&](auto&& f) {
        int it = 0;
        for (int u = u0; u < n_units; u += ustep) {
          const int tile = u / a.n_mblk;
          const Unit un{active[tv.u[tile]], u % a.n_mblk, tv.j0[tile]};
          for (int kc = 0; kc < a.kchunks; kc += KPS, ++it)   // one stage per KPS k-chunks
            if (!f(un, kc, it)) return;
        }
      };
      auto load_a = [&](const Unit& un, int kc, int it) {
        const int mb = un.mb, e = un.e, st = it % a.stages;
        uint8_t* sb = smem + (size_t)st * a.stage_bytes;
        // weights: when every expert has a single token tile (a.w_once) each
        // weight tile is read exactly once, so it is loaded evict-first
        // (Q4: packed nibbles of k-chunks kc, kc+1; the expanders build the A tiles)
        const int kx = DT == 8 ? kc * 128 : kc * 64;
        if (a.w_once) {
          tc::tma_load_3d_hint(sb, &tmA0.m, kx, mb * 128, e, &full[st], wpol);
          if (NM == 2) tc::tma_load_3d_hint(sb + A_BYTES, &tmA1.m, kx, mb * 128, e, &full[st], wpol);
        } else {
          tc::tma_load_3d(sb, &tmA0.m, kx, mb * 128, e, &full[st]);
          if (NM == 2) tc::tma_load_3d(sb + A_BYTES, &tmA1.m, kx, mb * 128, e, &full[st]);
        }
      };
      auto load_b = [&](const Unit& un, int kc, int it) {
        const int st = it % a.stages;
        uint8_t* sb = smem + (size_t)st * a.stage_bytes;
        const int by = a.tokb ? 0 : un.j0;   // decode: all token rows from row 0
#pragma unroll
        for (int q = 0; q < KPS; ++q) {
          uint8_t* bb = sb + NM * A_BYTES + q * NL * B_BYTES;
          tc::tma_load_2d(bb, &tmB0.m, (kc + q) * 128, by, &full[st]);
          if (NL == 2) tc::tma_load_2d(bb + B_BYTES, &tmB1.m, (kc + q) * 128, by, &full[st]);
        }
      };
      int pre = 0;   // iterations whose weights went out before the dependency wait
      if (MODE == DOWN) {
        for_iters([&](const Unit& un, int kc, int it) {
          if (it >= a.stages) return false;
          mbar_arrive_expect_tx(&full[it], bytes);
          load_a(un, kc, it);
          pre = it + 1;
          return true;
        });
        pdl_wait();
        pdl_launch();
        for_iters([&](const Unit& un, int kc, int it) {
          if (it >= pre) return false;
          load_b(un, kc, it);
          return true;
        });
        s_issued = pre;
      }
      for_iters([&](const Unit& un, int kc, int it) {
        if (*abort_flag) return false;
        if (it < pre) return true;
        const int st = it % a.stages;
        if (it >= a.stages && !mbar_wait(&empty[st], ((it / a.stages) - 1) & 1, kWaitNs)) {
          atomicOr(a.err, kErrTimeout); *abort_flag = 1; return false;
        }
        mbar_arrive_expect_tx(&full[st], bytes);
        load_a(un, kc, it);
        load_b(un, kc, it);
        Q4T(it, 0);
        s_issued = it + 1;
        return true;
      });
    }
  } else if (warp == 1) {
    // ------------------------- MMA issuer ---------------------------
    if (lane == 0) {
      // Q8: A = s8 weights, B = u8 low limb / s8 high limb.
      // Q4: A = u8 nibbles (0..15), B = s8 activations.
      uint32_t idesc[2];
      idesc[0] = tc::idesc_i8(128, NT, DT == 8, DT != 8);
      idesc[1] = tc::idesc_i8(128, NT, true, true);
      int ik = 0, ul = 0;                      // k-chunks consumed, units
      for (int u = u0; u < n_units && !*abort_flag; u += ustep, ++ul) {
        const int buf = ul & 1;
        if (ul >= 2 && !mbar_wait(&acc_empty[buf], ((ul >> 1) - 1) & 1, kWaitNs)) {
          atomicOr(a.err, kErrTimeout); *abort_flag = 1; break;
        }
        tc::fence_after_sync();
        const uint32_t dbase = tmem + buf * ACC;
        for (int kc = 0; kc < a.kchunks; ++kc, ++ik) {
          const int it = ik / KPS, st = it % a.stages, q = ik % KPS;   // stage and k-chunk within it
          const int ab = ik % AR;
          if (!mbar_wait(DT == 4 ? &afull[ab] : &full[st], DT == 4 ? (ik / AR) & 1 : (it / a.stages) & 1,
                         kWaitNs)) {
            atomicOr(a.err, kErrTimeout); *abort_flag = 1; break;
          }
          tc::fence_after_sync();
          if (threadIdx.x == 32 && q == 0) Q4T(it, 3);
          const uint8_t* sb = smem + (size_t)st * a.stage_bytes;
          const uint8_t* atile = DT == 4 ? aring + (size_t)ab * NM * A_BYTES : sb;
          const uint8_t* btile = sb + NM * A_BYTES + q * NL * B_BYTES;
          uint64_t da[NM], db[NL];
#pragma unroll
          for (int m = 0; m < NM; ++m) da[m] = ATM ? 0 : tc::sw128_desc(atile + m * A_BYTES);
#pragma unroll
          for (int l = 0; l < NL; ++l) db[l] = tc::sw128_desc(btile + l * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)            // 4 x 32 bytes of K per 128-byte chunk
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
              for (int l = 0; l < NL; ++l) {
                if (ATM)   // A: 32 TMEM columns per tile, 8 per 32-byte K step
                  tc::mma_i8_ts(dbase + (m * NL + l) * NT, tmem + ACOL + (ab * NM + m) * 32 + kk * 8,
                                db[l] + 2 * kk, idesc[l], (kc | kk) != 0);
                else
                  tc::mma_i8(dbase + (m * NL + l) * NT, da[m] + 2 * kk, db[l] + 2 * kk, idesc[l],
                             (kc | kk) != 0);
              }
          if (q == KPS - 1) tc::mma_commit(&empty[st]);   // stage free once its MMAs finish
          if (DT == 4) tc::mma_commit(&aempty[ab]);      // and the expanded A tiles
        }
        if (*abort_flag) break;
        tc::mma_commit(&acc_full[buf]);             // accumulator of this tile complete
      }
    }
  } else if (DT == 4 && warp >= kExpWarp0) {
    // ------------------- Q4 nibble expanders ------------------------
    // A stage holds, per matrix, 128 packed rows of 128 bytes (k-chunks kc and
    // kc+1, 128B-swizzled by the tensor copy: 16-byte chunk h of row r at
    // h ^ (r & 7)). For k-chunk q of the stage, packed 16-byte chunk c of row r
    // (= row bytes 64q + 16c) becomes two 16-byte chunks of the 128B-swizzled
    // u8 A tile: chunk 2c holds its 16 low nibbles, chunk 2c+1 its 16 high
    // nibbles (the activations use the same k order, q4_mma_pos). Thread ti
    // takes items ti + kExpThreads*i = (row, chunk): a warp covers 8 rows,
    // spread over all banks by the swizzle.
    const int ti = (warp - kExpWarp0) * 32 + lane;
    int ik = 0;
    for (int u = u0; u < n_units && !*abort_flag; u += ustep) {
      for (int kc = 0; kc < a.kchunks; ++kc, ++ik) {
        const int it = ik / KPS, st = it % a.stages, qk = ik % KPS, ab = ik % AR;
        if (!mbar_wait(&full[st], (it / a.stages) & 1, kWaitNs) ||
            (ik >= AR && !mbar_wait(&aempty[ab], ((ik / AR) - 1) & 1, kWaitNs))) {
          if (lane == 0) { atomicOr(a.err, kErrTimeout); *abort_flag = 1; }
          break;
        }
        if (ti == 0 && qk == 0) Q4T(it, 1);
        const uint8_t* stg = smem + (size_t)st * a.stage_bytes;
        if (ATM) {
          // warp = (lane quarter, part): part = matrix (gate/up) or column half
          // (down); row r's packed 64 bytes of this k-chunk -> 128 bytes = 32
          // TMEM columns (chunk 2c = columns 8c..8c+3, chunk 2c+1 = 8c+4..8c+7)
          const int quarter = warp & 3, part = (warp - kExpWarp0) >> 2, r = quarter * 32 + lane;
          const int m = NM == 2 ? part : 0;
          const uint8_t* prow = stg + m * A_BYTES + r * 128;
          const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + ACOL + (ab * NM + m) * 32;
          auto unpack = [&](int c, uint32_t* o) {
            const uint4 w = *reinterpret_cast<const uint4*>(prow + ((((qk << 2) + c) ^ (r & 7)) << 4));
            o[0] = w.x & 0x0F0F0F0Fu; o[1] = w.y & 0x0F0F0F0Fu; o[2] = w.z & 0x0F0F0F0Fu; o[3] = w.w & 0x0F0F0F0Fu;
            o[4] = (w.x >> 4) & 0x0F0F0F0Fu; o[5] = (w.y >> 4) & 0x0F0F0F0Fu;
            o[6] = (w.z >> 4) & 0x0F0F0F0Fu; o[7] = (w.w >> 4) & 0x0F0F0F0Fu;
          };
          if (NM == 2) {
            uint32_t o[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) unpack(c, o + 8 * c);
            tc::tmem_st32(trow, o);
          } else {
            uint32_t o[16];
#pragma unroll
            for (int c = 0; c < 2; ++c) unpack(2 * part + c, o + 8 * c);
            tc::tmem_st16(trow + 16 * part, o);
          }
          tc::tmem_wait_st();
          tc::fence_before_sync();          // TMEM stores -> the MMA thread after the barrier
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[ab]);
          if (ti == 0 && qk == KPS - 1) Q4T(it, 2);
          continue;
        }
        uint8_t* at = aring + (size_t)ab * NM * A_BYTES;
        // every packed chunk of this k-chunk is loaded before the first
        // expanded store: the compiler cannot move a shared load above a
        // shared store it may alias, so load/store pairs would each wait out
        // the load latency in turn
        constexpr int NI = 512 / (kExpWarps > 0 ? kExpThreads : 128);
        uint4 wv[NM][NI];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
          for (int i = 0; i < NI; ++i) {
            const int item = ti + kExpThreads * i, r = item >> 2, c = item & 3;
            wv[m][i] = *reinterpret_cast<const uint4*>(stg + m * A_BYTES + r * 128 +
                                                       ((((qk << 2) + c) ^ (r & 7)) << 4));
          }
#pragma unroll
        for (int m = 0; m < NM; ++m) {
#pragma unroll
          for (int i = 0; i < NI; ++i) {
            const int item = ti + kExpThreads * i, r = item >> 2, c = item & 3;
            const uint4 w = wv[m][i];
            uint8_t* dst = at + m * A_BYTES + r * 128;
            const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
            const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu,
                                        (w.z >> 4) & 0x0F0F0F0Fu, (w.w >> 4) & 0x0F0F0F0Fu);
            *reinterpret_cast<uint4*>(dst + (((2 * c) ^ (r & 7)) << 4)) = lo;
            *reinterpret_cast<uint4*>(dst + (((2 * c + 1) ^ (r & 7)) << 4)) = hi;
          }
        }
        tc::fence_proxy_async_smem();     // generic-proxy writes -> visible to the MMA
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[ab]);
        if (ti == 0 && qk == KPS - 1) Q4T(it, 2);
      }
    }
  } else {
    // ------------------------- epilogue -----------------------------
    const int q = warp & 3;                         // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;               // which 8-column chunks this warp takes (of kEpiPerQ)
    const int r = q * 32 + lane;                    // weight row within the 128-row block
    int ul = 0;
    for (int u = u0; u < n_units; u += ustep, ++ul) {
      const int buf = ul & 1;
      if (!mbar_wait(&acc_full[buf], (ul >> 1) & 1, kWaitNs)) {
        if (lane == 0) { atomicOr(a.err, kErrTimeout); *abort_flag = 1; }
        break;
      }
      tc::fence_after_sync();
      const int tile = u / a.n_mblk, mb = u % a.n_mblk;
      const int e = active[tv.u[tile]], j0 = tv.j0[tile], nt = tv.cnt[tile];
      const int n = mb * 128 + r;
      const uint8_t* ex = a.slab + (size_t)e * a.stride;
      const float sc0 = __ldg(reinterpret_cast<const float*>(ex + a.s0_off) + n);
      const float sc1 = NM == 2 ? __ldg(reinterpret_cast<const float*>(ex + a.s1_off) + n) : 0.f;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * ACC;
      // one (row n, sorted slot j) output from its raw accumulator words
      // as: the Q4 zero-point sum of slot j (Σa of its token for gate/up, Σh
      // of the slot for down), loaded by the caller
      auto emit = [&](const int j, const uint32_t (&raw)[NM * NL], const int as) {
        int dot[NM];
  #pragma unroll
        for (int m = 0; m < NM; ++m)
          dot[m] = NL == 2 ? (int)(raw[m * 2] + (raw[m * 2 + 1] << 8)) : (int)raw[m];
        if (DT == 4) {   // nibbles are stored +8: subtract 8 * Σ activation (exact mod 2^32)
  #pragma unroll
          for (int m = 0; m < NM; ++m) dot[m] = (int)((unsigned)dot[m] - 8u * (unsigned)as);
        }
        if (MODE == GATEUP) {
          const float g = fmul(div_qscale(dot[0], DT == 8), sc0);
          const float uu = fmul(div_qscale(dot[NM - 1], DT == 8), sc1);
          const float h = fmul(silu_ref(g), uu);
          const int ha = trunc_scale(h, S);
          if (DT == 8) {
            if (ha < -32768 || ha > 32767)
              range_fail(a.err, a.flags, __ldg(a.route + 2 + 2 * a.E_local + j) / a.topk);
            a.hs0[(size_t)j * a.F + n] = (uint8_t)(ha & 0xFF);
            a.hs1[(size_t)j * a.F + n] = (uint8_t)((ha >> 8) & 0xFF);
          } else {
            if (ha < -128 || ha > 127)
              range_fail(a.err, a.flags, __ldg(a.route + 2 + 2 * a.E_local + j) / a.topk);
            a.hs0[(size_t)j * a.F + q4_mma_pos(n)] = (uint8_t)(ha & 0xFF);
            // Σ h of slot j for the down projection's zero-point correction
            const int ws = __reduce_add_sync(0xffffffffu, ha);
            if (lane == 0) atomicAdd(a.hsum + j, ws);
          }
        } else {
          const float yv = fmul(div_qscale(dot[0], DT == 8), sc0);
          if (a.ep_on) {
            // expert parallel: the row goes straight to the rank owning the
            // slot's token, into its y buffer, over NVLink
            const int sl = __ldg(a.route + 2 + 2 * a.E_local + j);
            const int per = a.topk * a.ep.T_local;
            const int owner = sl / per;
            float* yo = reinterpret_cast<float*>(__ldg(reinterpret_cast<const unsigned long long*>(a.ep.base) + owner) +
                                                 a.ep.y_off);
            yo[(size_t)(sl - owner * per) * a.rows + n] = yv;
          } else {
            a.ys[(size_t)j * a.rows + n] = yv;
          }
        }
      };
      if (MODE == GATEUP && a.tokb) {
        // decode: B held all T token rows, so accumulator column t is token t;
        // each routed slot j of this expert reads its token's column
        for (int jj = half; jj < nt; jj += kEpiPerQ) {
          const int j = j0 + jj;
          const int t = __ldg(a.route + 2 + 2 * a.E_local + j) / a.topk;   // warp-uniform
          uint32_t v[NM * NL][8], raw[NM * NL];
#pragma unroll
          for (int x = 0; x < NM * NL; ++x) tc::tmem_ld8(tbase + x * NT + (t & ~7), v[x]);
          tc::tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < NM * NL; ++x) {
            raw[x] = v[x][0];
#pragma unroll
            for (int c = 1; c < 8; ++c) if ((t & 7) == c) raw[x] = v[x][c];
          }
          // decode gate/up: the token's Σa (Q4), through the slot's token index
          emit(j, raw, DT == 4 ? __ldg(a.xsum + __ldg(a.route + 2 + 2 * a.E_local + j) / a.topk) : 0);
        }
      } else {
        for (int c0 = 8 * half; c0 < nt; c0 += 8 * kEpiPerQ) {
          uint32_t v[NM * NL][8];
#pragma unroll
          for (int x = 0; x < NM * NL; ++x) tc::tmem_ld8(tbase + x * NT + c0, v[x]);
          // the group's 8 zero-point sums, loaded together before any of its
          // stores (the stores could alias them, so the compiler keeps loads
          // after earlier stores): sorted-slot Σa for gate/up (staged by the
          // gather), Σh for down (written by the gate/up kernel); through L2,
          // as the producing kernel may have finished only under this launch
          int asv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            asv[i] = (DT == 4 && c0 + i < nt) ? __ldcg((MODE == GATEUP ? a.xsum_s : a.hsum) + j0 + c0 + i) : 0;
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int jj = c0 + i;
            if (jj >= nt) break;
            uint32_t raw[NM * NL];
#pragma unroll
            for (int x = 0; x < NM * NL; ++x) raw[x] = v[x][i];
            emit(j0 + jj, raw, asv[i]);
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  __syncthreads();
  if (MODE == DOWN && a.ep_on && threadIdx.x == 0) {
    // The barrier orders the CTA's peer stores before this thread's system
    // fence; the last CTA to arrive then raises this rank's combine flag at
    // every rank (release), so a rank that sees the flag sees the rows.
    // When a token was marked out of range the exact fix-up pass that
    // follows raises them instead, after its own rows.
    __threadfence_system();
    int* counter = reinterpret_cast<int*>(a.ep.base_local + kEpCounter);
    if (atomicAdd(counter, 1) == (int)gridDim.x - 1) {
      *counter = 0;
      if (!(a.flags && *reinterpret_cast<volatile int*>(a.flags))) ep_raise_combine(a.ep);
    }
  }
  if (threadIdx.x == 0 && s_abort) {
    // let the tensor copies still in flight land before the CTA's smem goes away
    for (int it = max(0, s_issued - a.stages); it < s_issued; ++it)
      mbar_wait(&full[it % a.stages], (it / a.stages) & 1, kWaitNs);
  }
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TCOLS);
  }
  MOE_TL_END(MODE == GATEUP ? kTlGateup : kTlDown);
}

}  // namespace mm
}  // namespace moe

// ===========================================================================
// host side
// ===========================================================================
namespace moe {
namespace mm {

// Gather the routed tokens' activation rows into expert-sorted order:
// row j of the output planes = token slot_list[j] / topk (B operand rows);
// for Q4 also xsum_s[j] = that token's Σ activation (the zero-point term the
// gate/up epilogue subtracts). One warp per row, 16-byte copies, rows
// grid-strided over the CTAs.
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint8_t* __restrict__ xact, int act_stride, int D,
                                                          int nplanes, const int* __restrict__ route, int E_local,
                                                          int topk, uint8_t* __restrict__ xs0,
                                                          uint8_t* __restrict__ xs1, const int* __restrict__ xsum,
                                                          int* __restrict__ xsum_s) {
  MOE_TL_START(kTlGather);
  MOE_TL_END(kTlGather);
  pdl_wait();
  pdl_launch();
  const RouteView r = route_view(const_cast<int*>(route), E_local);
  const int J = r.exp_off[*r.n_active];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int n16 = D / 16;
  for (int j = blockIdx.x * 8 + w; j < J; j += gridDim.x * 8) {
    const int t = r.slot_list[j] / topk;
    const uint4* src = reinterpret_cast<const uint4*>(xact + (size_t)t * act_stride);
    uint4* d0 = reinterpret_cast<uint4*>(xs0 + (size_t)j * D);
    for (int i = lane; i < n16; i += 32) d0[i] = __ldg(src + i);
    if (nplanes == 2) {
      uint4* d1 = reinterpret_cast<uint4*>(xs1 + (size_t)j * D);
      for (int i = lane; i < n16; i += 32) d1[i] = __ldg(src + n16 + i);
    } else if (lane == 0) {
      xsum_s[j] = __ldg(xsum + t);
    }
  }
}

template <int DT, int MODE, int NT>
static bool launch_kernel(const TMap& a0, const TMap& a1, const TMap& b0, const TMap& b1, Args a, int grid,
                          cudaStream_t st) {
  constexpr int NM = MODE == GATEUP ? 2 : 1, NL = DT == 8 ? 2 : 1;
  a.stage_bytes = NM * 128 * 128 + (DT == 4 ? kQ4KPerStage : 1) * NL * NT * 128;
  const int aring = (DT == 4 && !q4_a_in_tmem(DT, NT)) ? q4_aring_depth(NT) * NM * 128 * 128 + 1024 : 0;
  const int budget = 220 * 1024 / ctas_for(DT, NT) - aring;
  a.stages = (budget - 1024 - 256) / a.stage_bytes;
  if (a.stages > 8) a.stages = 8;
  if (a.stages < 2) return false;
  const size_t smem = (size_t)a.stages * a.stage_bytes + 1024 + 16 * (size_t)a.stages + 32 +
                      16 * (DT == 4 ? q4_aring_depth(NT) : 2) + aring;
  auto k = moe_mma_kernel<DT, MODE, NT>;
  static size_t attr = 0;
  if (smem > attr) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return false;
    attr = smem;
  }
  return launch_pdl(k, dim3(grid), dim3(cta_threads(DT, NT)), smem, st, a0, a1, b0, b1, a) == cudaSuccess;
}

}  // namespace mm

// ---- public launchers ------------------------------------------------------

// Slots per tile: the smallest tile that holds a decode expert's slots; for
// Q4 prefill 128 (two 128-column accumulators, double-buffered, fill TMEM at
// one CTA per SM; weight blocks are re-read once per tile, so wider is better).
int mma_tile_n(int T, int dtype) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  return dtype == 3 && T > 256 ? 128 : 64;
}

// Q8: K dimensions in 128-element chunks; Q4: two chunks per pipeline stage.
bool mma_supported(const LayerDev& L) {
  const int kq = L.dtype == 3 ? 128 * mm::kQ4KPerStage : 128;
  return (L.dtype == 2 || L.dtype == 3) && L.D % kq == 0 && L.F % kq == 0 && L.D % 128 == 0 &&
         L.F % 128 == 0 && mm::encoder() != nullptr;
}

void launch_mma_gather(const LayerDev& L, const Workspace& ws, int T, int nt, cudaStream_t st) {
  if (T <= nt) return;   // decode: the GEMM reads the token rows directly
  const int E_local = L.e_end - L.e_begin, TK = T * L.topk;
  const int rows_per_cta = 8, cap = 8 * mm::sms();
  int grid = (TK + rows_per_cta - 1) / rows_per_cta;
  if (grid > cap) grid = cap;
  launch_pdl(mm::gather_rows_kernel, dim3(grid), dim3(256), 0, st, ws.xact, 2 * L.D, L.D, L.dtype == 2 ? 2 : 1,
             ws.route, E_local, L.topk, ws.xs0, ws.xs1, (const int*)ws.xsum, ws.xsum_s);
}

#define NT_SWITCH(nt, CALL) \
  switch (nt) {             \
    case 16: { constexpr int NT = 16; CALL; } break; \
    case 32: { constexpr int NT = 32; CALL; } break; \
    default: { constexpr int NT = 64; CALL; } break; \
  }
#define NT_SWITCH_Q4(nt, CALL) \
  switch (nt) {             \
    case 16: { constexpr int NT = 16; CALL; } break; \
    case 32: { constexpr int NT = 32; CALL; } break; \
    case 64: { constexpr int NT = 64; CALL; } break; \
    default: { constexpr int NT = 128; CALL; } break; \
  }

bool launch_mma_gateup(const LayerDev& L, const Workspace& ws, int T, int nt, int* err, cudaStream_t st) {
  const int E_local = L.e_end - L.e_begin, TK = T * L.topk, cap = ws.cap_T * ws.cap_K;
  mm::TMap a0, a1, b0, b1;
  // decode (every expert's slots fit one tile): B = the T token rows as they
  // are (lo plane, then the hi plane D bytes further; rows 2D apart), no gather
  const bool tokb = T <= nt;
  bool mapped;
  if (tokb)
    mapped = mm::map_rows(b0, ws.xact, L.D, ws.cap_T, nt, 2 * L.D) &&
             mm::map_rows(b1, ws.xact + (L.dtype == 2 ? L.D : 0), L.D, ws.cap_T, nt, 2 * L.D);
  else
    mapped = mm::map_rows(b0, ws.xs0, L.D, cap, nt) &&
             mm::map_rows(b1, L.dtype == 2 ? ws.xs1 : ws.xs0, L.D, cap, nt);
  if (!mapped || !mm::map_weights(a0, L, L.gq_off, L.D, L.F) || !mm::map_weights(a1, L, L.uq_off, L.D, L.F))
    return false;
  mm::Args a{};
  a.rows = L.F; a.kchunks = L.D / 128; a.n_mblk = L.F / 128;
  a.route = ws.route; a.E_local = E_local; a.TK = TK; a.max_tiles = route_max_tiles(TK, E_local, nt);
  a.slab = L.slab; a.stride = L.expert_stride; a.s0_off = L.gs_off; a.s1_off = L.us_off;
  a.F = L.F; a.hs0 = ws.hs0; a.hs1 = ws.hs1; a.err = err; a.flags = ws.xbad;
  a.xsum = ws.xsum; a.hsum = ws.hsum; a.xsum_s = ws.xsum_s;
  a.topk = L.topk; a.tokb = tokb; a.w_once = T <= nt && mm::evict_first_on();
  const int units = a.max_tiles * a.n_mblk, gc = mm::grid_ctas(L.dtype == 2 ? 8 : 4, nt);
  const int grid = units < gc ? units : gc;
  bool ok = false;
  if (L.dtype == 2) { NT_SWITCH(nt, (ok = mm::launch_kernel<8, mm::GATEUP, NT>(a0, a1, b0, b1, a, grid, st))); }
  else { NT_SWITCH_Q4(nt, (ok = mm::launch_kernel<4, mm::GATEUP, NT>(a0, a1, b0, b0, a, grid, st))); }
  return ok;
}

bool launch_mma_down(const LayerDev& L, const Workspace& ws, int T, int nt, float* ys, int* err, cudaStream_t st,
                     const EpView* ep) {
  const int E_local = L.e_end - L.e_begin, TK = T * L.topk, cap = ws.cap_T * ws.cap_K;
  mm::TMap a0, b0, b1;
  if (!mm::map_weights(a0, L, L.dq_off, L.F, L.D) || !mm::map_rows(b0, ws.hs0, L.F, cap, nt) ||
      !mm::map_rows(b1, L.dtype == 2 ? ws.hs1 : ws.hs0, L.F, cap, nt))
    return false;
  mm::Args a{};
  a.rows = L.D; a.kchunks = L.F / 128; a.n_mblk = L.D / 128;
  a.route = ws.route; a.E_local = E_local; a.TK = TK; a.max_tiles = route_max_tiles(TK, E_local, nt);
  a.slab = L.slab; a.stride = L.expert_stride; a.s0_off = L.ds_off;
  a.ys = ys; a.T = T; a.topk = L.topk; a.flags = ws.xbad;
  a.err = err;
  a.xsum = ws.xsum; a.hsum = ws.hsum; a.ep_on = ep != nullptr;
  a.w_once = T <= nt && mm::evict_first_on();
  if (ep) a.ep = *ep;
  const int units = a.max_tiles * a.n_mblk, gc = mm::grid_ctas(L.dtype == 2 ? 8 : 4, nt);
  const int grid = units < gc ? units : gc;
  bool ok = false;
  if (L.dtype == 2) { NT_SWITCH(nt, (ok = mm::launch_kernel<8, mm::DOWN, NT>(a0, a0, b0, b1, a, grid, st))); }
  else { NT_SWITCH_Q4(nt, (ok = mm::launch_kernel<4, mm::DOWN, NT>(a0, a0, b0, b0, a, grid, st))); }
  return ok;
}

// combine from expert-sorted y rows (prefill / non-fused path)
// Scalar form (any D, any alignment of xres/out): one thread per output.
__global__ void combine_sorted_scalar_kernel(const float* __restrict__ ys, const int* __restrict__ slot_pos,
                                             const float* __restrict__ p, const int* __restrict__ idx,
                                             const float* xres, float* out, int T, int D, int K, int seq,
                                             const HostOut ho) {
  pdl_wait();
  pdl_launch();
  const long q = (long)blockIdx.x * blockDim.x + threadIdx.x;
  publish_host(ho, q, (long)gridDim.x * blockDim.x);
  if (q >= (long)T * D) return;
  const int t = (int)(q / D), n = (int)(q % D);
  float acc = seq ? xres[q] : 0.0f;
  for (int k = 0; k < K; ++k) {
    const int s = t * K + k;
    acc = fadd(acc, fmul(p[s], idx[s] < 0 ? 0.0f : ys[(size_t)slot_pos[s] * D + n]));
  }
  out[q] = seq ? acc : fadd(xres[q], acc);
}

// One thread per 4 consecutive outputs of a token (D % 4 == 0, 16-byte
// aligned rows): the token's routing words once, then 16-byte loads of its K
// slot rows.
__global__ void combine_sorted_kernel(const float* __restrict__ ys, const int* __restrict__ slot_pos,
                                      const float* __restrict__ p, const int* __restrict__ idx,
                                      const float* xres, float* out, int T, int D, int K, int seq,
                                      const HostOut ho) {
  MOE_TL_START(kTlCombine);
  pdl_wait();
  pdl_launch();
  const long q = (long)blockIdx.x * blockDim.x + threadIdx.x;
  publish_host(ho, q, (long)gridDim.x * blockDim.x);
  const int D4 = D / 4;
  if (q >= (long)T * D4) return;
  const int t = (int)(q / D4), n = (int)(q % D4) * 4;
  const size_t o = (size_t)t * D + n;
  // seq: accumulate into the residual in k order (model.c:188), else add the
  // k-ordered sum to it (test_model_trace.c:513,517)
  const float4 xr = *reinterpret_cast<const float4*>(xres + o);
  float4 acc = seq ? xr : make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [&](float pk, float4 y) {
    acc.x = fadd(acc.x, fmul(pk, y.x));
    acc.y = fadd(acc.y, fmul(pk, y.y));
    acc.z = fadd(acc.z, fmul(pk, y.z));
    acc.w = fadd(acc.w, fmul(pk, y.w));
  };
  constexpr int KF = 8;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  if (K <= KF) {
    // all slots' routing words first, then all their y values: two dependent
    // load rounds instead of 2K; the sum keeps the k order
    int js[KF];
    float ps[KF];
    float4 yv[KF];
#pragma unroll
    for (int k = 0; k < KF; ++k) {
      js[k] = -1;
      ps[k] = 0.f;
      if (k < K) {
        const int s = t * K + k;
        const int e = __ldg(idx + s), j = __ldg(slot_pos + s);
        ps[k] = __ldg(p + s);
        js[k] = e < 0 ? -1 : j;
      }
    }
    // a slot with no expert (idx < 0) adds p * 0, as combine_kernel
#pragma unroll
    for (int k = 0; k < KF; ++k)
      yv[k] = js[k] >= 0 ? __ldg(reinterpret_cast<const float4*>(ys + (size_t)js[k] * D + n)) : zero;
#pragma unroll
    for (int k = 0; k < KF; ++k)
      if (k < K) add(ps[k], yv[k]);
  } else {
    for (int k = 0; k < K; ++k) {
      const int s = t * K + k;
      add(p[s], idx[s] < 0 ? zero : *reinterpret_cast<const float4*>(ys + (size_t)slot_pos[s] * D + n));
    }
  }
  if (!seq) {
    acc.x = fadd(xr.x, acc.x);
    acc.y = fadd(xr.y, acc.y);
    acc.z = fadd(xr.z, acc.z);
    acc.w = fadd(xr.w, acc.w);
  }
  *reinterpret_cast<float4*>(out + o) = acc;
  MOE_TL_END(kTlCombine);
}

void launch_combine_sorted(const float* ys, const int* slot_pos, const float* p, const int* idx,
                           const float* xres, float* out, int T, int D, int K, cudaStream_t st, bool seq_residual,
                           const HostOut& ho) {
  if (D % 4 || ((uintptr_t)xres | (uintptr_t)out | (uintptr_t)ys) % 16) {
    const long n1 = (long)T * D;
    if (n1 > 0)
      launch_pdl(combine_sorted_scalar_kernel, dim3((unsigned)((n1 + 255) / 256)), dim3(256), 0, st, ys, slot_pos, p,
                 idx, xres, out, T, D, K, seq_residual ? 1 : 0, ho);
    return;
  }
  const long total = (long)T * (D / 4);
  if (total <= 0) return;
  launch_pdl(combine_sorted_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, ys, slot_pos, p, idx, xres,
             out, T, D, K, seq_residual ? 1 : 0, ho);
}

// Expert-parallel output: slot-ordered rows of this rank's slots, zeros for
// slots whose expert lives on another rank (so a sum over ranks is exact).
__global__ void unsort_rows_kernel(const float* __restrict__ ys, const int* __restrict__ slot_pos,
                                   const int* __restrict__ idx, int e_begin, int e_end,
                                   float* __restrict__ y_slots, int D) {
  const int s = blockIdx.x;
  pdl_wait();
  pdl_launch();
  const int e = idx[s];
  float4* dst = reinterpret_cast<float4*>(y_slots + (size_t)s * D);
  if (e < e_begin || e >= e_end) {
    for (int i = threadIdx.x; i < D / 4; i += blockDim.x) dst[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  const float4* src = reinterpret_cast<const float4*>(ys + (size_t)slot_pos[s] * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) dst[i] = src[i];
}

void launch_unsort_rows(const LayerDev& L, const Workspace& ws, int T, float* y_slots, cudaStream_t st) {
  launch_pdl(unsort_rows_kernel, dim3(T * L.topk), dim3(128), 0, st, ws.y, ws.slot_pos, ws.topk_idx, L.e_begin,
             L.e_end, y_slots, L.D);
}

#ifdef MOE_TIMELINE
void q4_trace_read(long long* out) { cudaMemcpyFromSymbol(out, mm::g_q4_trace, sizeof(mm::g_q4_trace)); }
#endif
MOE_TL_IO(moe_mma)

}  // namespace moe
