/*
 * moe_oracle.c — CPU restatement of moe.cc's MoE expert-FFN path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for libmoe_cuda.so: it
 * is compiled into oracle/liboracle.so and loaded by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg. Nothing in the
 * product links or calls it.
 *
 * Every function restates one piece of the reference's algorithm in my own
 * code and names the reference file:line it follows. It is pinned against
 * the reference itself: oracle/ref_shim.c compiles the reference's own
 * kernels.c and test_model_trace.c (from their sources) into
 * oracle/_ref/libmoe_ref.so, and tests compare the two, plus committed golden
 * vectors made from both (tests/golden/make_golden.py).
 *
 * Build: gcc -O3 -fopenmp -ffp-contract=off (no -ffast-math, no -march):
 * float arithmetic is IEEE single with one rounding per operation and no FMA,
 * the same as the reference's gcc -O2 x86-64 build (Makefile:2-3). The
 * activation truncation of kernels.c is hoisted out of the row loop; it is
 * the same value for every row, so results are unchanged.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* (int32_t)(a * scale): kernels.c:66 (Q8, 127.0f) and :113 (Q4, 7.0f). */
static void trunc_row(const float* a, int K, float scale, int32_t* out) {
  for (int k = 0; k < K; ++k) out[k] = (int32_t)(a[k] * scale);
}

/* Integer dot with two's-complement wrap: the reference's int32 `dot_i32 +=`
 * (kernels.c:67, :122-125). Done in uint32 so the wrap is defined. */
static int32_t dot_q8(const int32_t* aq, const int8_t* w, int K) {
  uint32_t acc = 0;
  for (int k = 0; k < K; ++k) acc += (uint32_t)(aq[k] * (int32_t)w[k]);
  return (int32_t)acc;
}

static int32_t dot_q4(const int32_t* aq, const uint8_t* w, int K) {
  uint32_t acc = 0;
  for (int k = 0; k < K; k += 2) {
    const uint8_t b = w[k >> 1];
    acc += (uint32_t)(aq[k] * ((int32_t)(b & 0xF) - 8));      /* kernels.c:111 */
    acc += (uint32_t)(aq[k + 1] * ((int32_t)(b >> 4) - 8));   /* kernels.c:112 */
  }
  return (int32_t)acc;
}

/* matmul_f32_q8, kernels.c:51-74: C[m,n] = ((float)dot / 127f) * s[n]. */
int orc_matmul_q8(const float* A, const int8_t* Bq, const float* Bs, float* C,
                  int M, int N, int K) {
  int32_t* aq = (int32_t*)malloc(sizeof(int32_t) * (size_t)(K > 0 ? K : 1));
  if (!aq) return -1;
  for (int m = 0; m < M; ++m) {
    trunc_row(A + (size_t)m * K, K, 127.0f, aq);
    for (int n = 0; n < N; ++n) {
      const int32_t d = dot_q8(aq, Bq + (size_t)n * K, K);
      C[(size_t)m * N + n] = ((float)d / 127.0f) * Bs[n];          /* :71 */
    }
  }
  free(aq);
  return 0;
}

/* matmul_f32_q4, kernels.c:96-128 (even K only; the reference reads one
 * byte past the packed row for odd K, kernels.c:108,116). */
int orc_matmul_q4(const float* A, const uint8_t* Bq, const float* Bs, float* C,
                  int M, int N, int K) {
  if (K & 1) return -1;
  int32_t* aq = (int32_t*)malloc(sizeof(int32_t) * (size_t)(K > 0 ? K : 1));
  if (!aq) return -1;
  for (int m = 0; m < M; ++m) {
    trunc_row(A + (size_t)m * K, K, 7.0f, aq);
    for (int n = 0; n < N; ++n) {
      const int32_t d = dot_q4(aq, Bq + (size_t)n * (K / 2), K);
      C[(size_t)m * N + n] = ((float)d / 7.0f) * Bs[n];            /* :126 */
    }
  }
  free(aq);
  return 0;
}

/* fp32 branch of matmul_adaptive (kernels.c:153-165) and the router's
 * matmul_f32 (test_model_trace.c:213-227): one sequential fp32 sum per
 * output, mul then add, each rounded. */
void orc_matmul_f32(const float* A, const float* W, float* C, int M, int N, int K) {
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      const float* a = A + (size_t)m * K;
      const float* w = W + (size_t)n * K;
      float acc = 0.0f;
      for (int k = 0; k < K; ++k) acc += a[k] * w[k];
      C[(size_t)m * N + n] = acc;
    }
}

/* topk_desc, test_model_trace.c:275-288: insertion into a descending list;
 * strict '>' keeps the lower expert index on ties; NaN is never inserted. */
void orc_topk_desc(const float* x, int E, int k, int* idx, float* val) {
  for (int i = 0; i < k; ++i) { val[i] = -INFINITY; idx[i] = -1; }
  for (int e = 0; e < E; ++e) {
    const float v = x[e];
    int pos = -1;
    for (int i = 0; i < k; ++i) if (v > val[i]) { pos = i; break; }
    if (pos < 0) continue;
    for (int j = k - 1; j > pos; --j) { val[j] = val[j - 1]; idx[j] = idx[j - 1]; }
    val[pos] = v; idx[pos] = e;
  }
}

/* softmax over the selected logits, test_model_trace.c:481-487. */
void orc_topk_softmax(float* v, int k) {
  float mx = v[0];
  for (int i = 1; i < k; ++i) if (v[i] > mx) mx = v[i];
  float sum = 0.0f;
  for (int i = 0; i < k; ++i) { v[i] = expf(v[i] - mx); sum += v[i]; }
  const float inv = 1.0f / (sum + 1e-9f);
  for (int i = 0; i < k; ++i) v[i] *= inv;
}

/*
 * The MoE block of layer_forward_f32, test_model_trace.c:463-517, with the
 * quantised-expert branch (:494-503):
 *   logits = x_norm2 · Wrᵀ (+ b)                  :464-468
 *   per token: topk_desc, softmax over the top-k  :480-487
 *   per (t,i): g = Wg·x; g = silu(g); u = Wu·x; g *= u; y = Wd·g  :496-503
 *              moe_out[t] += p * y                :513
 *   x_out = x_after + moe_out                     :517
 * Expert weights are contiguous per projection: gq [E][F][D or D/2],
 * uq like gq, dq [E][D][F or F/2]; scales gs/us [E][F], ds [E][D].
 * dtype 2 = Q8, 3 = Q4. Outputs: x_out [T][D]; optional idx/p [T][topk],
 * logits [T][E]. Tokens are independent, so they run in parallel (OpenMP);
 * each token's arithmetic is exactly sequential as in the reference.
 */
int orc_moe_block(const float* x_norm2, const float* x_after, float* x_out,
                  int T, int D, int E, int topk, int F,
                  const float* router_w, const float* router_b, int dtype,
                  const void* gq, const float* gs, const void* uq,
                  const float* us, const void* dq, const float* ds,
                  int* idx_out, float* p_out, float* logits_out) {
  if (dtype != 2 && dtype != 3) return -1;
  if (dtype == 3 && ((D & 1) || (F & 1))) return -1;
  const size_t gu_row = dtype == 2 ? (size_t)D : (size_t)D / 2;
  const size_t d_row = dtype == 2 ? (size_t)F : (size_t)F / 2;
  int err = 0;
#pragma omp parallel for schedule(dynamic, 1)
  for (int t = 0; t < T; ++t) {
    float* logits = (float*)malloc(sizeof(float) * (size_t)E);
    int* idx = (int*)malloc(sizeof(int) * (size_t)topk);
    float* val = (float*)malloc(sizeof(float) * (size_t)topk);
    float* g = (float*)malloc(sizeof(float) * (size_t)F);
    float* u = (float*)malloc(sizeof(float) * (size_t)F);
    float* y = (float*)malloc(sizeof(float) * (size_t)D);
    float* acc = (float*)malloc(sizeof(float) * (size_t)D);
    if (!logits || !idx || !val || !g || !u || !y || !acc) {
#pragma omp atomic write
      err = 1;
    } else {
      const float* x = x_norm2 + (size_t)t * D;
      orc_matmul_f32(x, router_w, logits, 1, E, D);
      if (router_b) for (int e = 0; e < E; ++e) logits[e] += router_b[e];
      if (logits_out) memcpy(logits_out + (size_t)t * E, logits, sizeof(float) * (size_t)E);
      orc_topk_desc(logits, E, topk, idx, val);
      orc_topk_softmax(val, topk);
      for (int q = 0; q < D; ++q) acc[q] = 0.0f;
      for (int i = 0; i < topk; ++i) {
        const int e = idx[i];
        const float p = val[i];
        if (e < 0) {
          /* fewer than topk logits that are neither NaN nor -inf: the
           * reference indexes expert -1 (out of bounds, undefined). Its p is
           * then 0 (a finite maximum exists) or NaN (none does), so p * y is
           * 0 or NaN whatever that memory holds; restated as p * 0. */
          for (int q = 0; q < D; ++q) acc[q] += p * 0.0f;
          continue;
        }
        if (dtype == 2) {
          orc_matmul_q8(x, (const int8_t*)gq + (size_t)e * F * gu_row, gs + (size_t)e * F, g, 1, F, D);
        } else {
          orc_matmul_q4(x, (const uint8_t*)gq + (size_t)e * F * gu_row, gs + (size_t)e * F, g, 1, F, D);
        }
        for (int q = 0; q < F; ++q) g[q] = g[q] / (1.0f + expf(-g[q]));   /* silu_f32 :229-236 */
        if (dtype == 2) {
          orc_matmul_q8(x, (const int8_t*)uq + (size_t)e * F * gu_row, us + (size_t)e * F, u, 1, F, D);
        } else {
          orc_matmul_q4(x, (const uint8_t*)uq + (size_t)e * F * gu_row, us + (size_t)e * F, u, 1, F, D);
        }
        for (int q = 0; q < F; ++q) g[q] *= u[q];                            /* :501 */
        if (dtype == 2) {
          orc_matmul_q8(g, (const int8_t*)dq + (size_t)e * D * d_row, ds + (size_t)e * D, y, 1, D, F);
        } else {
          orc_matmul_q4(g, (const uint8_t*)dq + (size_t)e * D * d_row, ds + (size_t)e * D, y, 1, D, F);
        }
        for (int q = 0; q < D; ++q) acc[q] += p * y[q];                      /* :513 */
      }
      const float* xa = x_after + (size_t)t * D;
      float* xo = x_out + (size_t)t * D;
      for (int q = 0; q < D; ++q) xo[q] = xa[q] + acc[q];                   /* :517 */
      if (idx_out) memcpy(idx_out + (size_t)t * topk, idx, sizeof(int) * (size_t)topk);
      if (p_out) memcpy(p_out + (size_t)t * topk, val, sizeof(float) * (size_t)topk);
    }
    free(logits); free(idx); free(val); free(g); free(u); free(y); free(acc);
  }
  return err ? -1 : 0;
}

/* Rowwise quantisers, export.py:23-27 (_rowwise_q8) and :29-36 (_rowwise_q4):
 * s = max(max|row|, 1e-8) / 127 (or / 7) in fp32; q = round-half-even(w / s)
 * with an fp32 divide; Q4 clamps to [-8,7], adds 8 and packs column 2j in the
 * low nibble of byte j, column 2j+1 in the high nibble. */
void orc_quantize_q8(const float* W, int rows, int cols, int8_t* q, float* s) {
  for (int r = 0; r < rows; ++r) {
    const float* w = W + (size_t)r * cols;
    float amax = 0.0f;
    for (int c = 0; c < cols; ++c) { const float a = fabsf(w[c]); if (a > amax) amax = a; }
    if (!(amax >= 1e-8f)) amax = 1e-8f;   /* clamp(min=1e-8) */
    const float sc = amax / 127.0f;
    s[r] = sc;
    for (int c = 0; c < cols; ++c) q[(size_t)r * cols + c] = (int8_t)(int32_t)rintf(w[c] / sc);
  }
}

int orc_quantize_q4(const float* W, int rows, int cols, uint8_t* q, float* s) {
  if (cols & 1) return -1;
  for (int r = 0; r < rows; ++r) {
    const float* w = W + (size_t)r * cols;
    float amax = 0.0f;
    for (int c = 0; c < cols; ++c) { const float a = fabsf(w[c]); if (a > amax) amax = a; }
    if (!(amax >= 1e-8f)) amax = 1e-8f;
    const float sc = amax / 7.0f;
    s[r] = sc;
    for (int c = 0; c < cols; c += 2) {
      float v0 = rintf(w[c] / sc), v1 = rintf(w[c + 1] / sc);
      v0 = v0 < -8.0f ? -8.0f : (v0 > 7.0f ? 7.0f : v0);
      v1 = v1 < -8.0f ? -8.0f : (v1 > 7.0f ? 7.0f : v1);
      const uint8_t lo = (uint8_t)((int)v0 + 8), hi = (uint8_t)((int)v1 + 8);
      q[(size_t)r * (cols / 2) + c / 2] = (uint8_t)(lo | (hi << 4));
    }
  }
  return 0;
}

/* Seeded N(0, std) stream used to make the benchmark's synthetic inputs:
 * element i of stream `seed` is splitmix64 at counters 2i and 2i+1 -> two
 * uniforms in [0,1) (53 bits) -> Box-Muller in double -> float. This is the
 * same stream the product draws on the device and host, restated here so the
 * reference arm of the benchmark builds its inputs without loading the
 * product library. Not part of the reference's algorithm (its inputs are a
 * checkpoint); pinned equal to the product's stream by tests/. */
static uint64_t orc_splitmix_at(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

void orc_synth_normal(uint64_t seed, uint64_t offset, size_t n, float std, float* out) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i) {
    const uint64_t j = offset + (uint64_t)i;
    const double u1 = (double)(orc_splitmix_at(seed, 2 * j) >> 11) * 0x1.0p-53;
    const double u2 = (double)(orc_splitmix_at(seed, 2 * j + 1) >> 11) * 0x1.0p-53;
    const double z = sqrt(-2.0 * log(1.0 - u1)) * cos(6.283185307179586 * u2);
    out[i] = (float)(z * (double)std);
  }
}
