/*
 * moe_host.c — the C host driver of include/moe_host.h: KV-cached, batched
 * decode with fp32 attention on the CPU and the MoE block on the GPU.
 *
 * CPU arithmetic is written to give the reference's results bit for bit
 * (compiled with -ffp-contract=off, no fast-math, so every product and sum
 * is a separately rounded IEEE operation in the order shown):
 *   matmul_f32 (test_model_trace.c:213-227): each output is one sequential
 *     chain acc = 0; acc += a[k]*w[k] for k = 0..K-1. Parallelism is over
 *     outputs only: 16 outputs per pass in 8-wide AVX2 lanes where the CPU
 *     has AVX2, else four scalar chains per pass.
 *   rmsnorm_forward_f32 (:241-255): msq sequential, msq /= D,
 *     inv = 1/sqrtf(msq + eps), y = (x*inv)*w.
 *   per-head Q/K RMSNorm (:371-392): inv = 1/sqrtf(msq/hd + eps),
 *     y = (v*inv)*w.
 *   RoPE (:297-336): inv_freq[i] = powf(theta, (-2*i)/hd),
 *     angle = pos*inv_freq[i], pairs (i, i+hd/2).
 *   attention (:394-420): scores dot*scale in key order, max, expf sum,
 *     1/(sum+1e-9), then out[d] += p*v[d] in key order. The reference runs
 *     every key of the prefix with the later ones masked to -inf; those add
 *     exactly 0 to the sum and 0*v to the output, so stopping at the
 *     query's own position gives the same values.
 * glibc's expf/sqrtf/powf/cosf/sinf are called as the reference calls them.
 */
#define _POSIX_C_SOURCE 200809L
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <cuda_runtime.h>
#include <immintrin.h>
#include <omp.h>

#include "../../include/moe_cuda.h"
#include "../../include/moe_host.h"

typedef struct {
  MhLayerWeights w;
} Layer;

struct MhModel {
  MhConfig c;
  int batch, max_ctx, moe_base, pos;
  int Dq, Dkv;
  Layer* layers;
  const float *tok_emb, *final_norm_w, *lm_head;
  float** owned;                 /* host allocations freed with the model */
  int n_owned, cap_owned;
  float *kc, *vc;                /* [layer][batch][max_ctx][Dkv] */
  /* per-step scratch, grown to the step's rows */
  int cap_rows;
  int pinned_rows;                 /* x, xa, xn2 came from cudaHostAlloc */
  float *xn1, *q, *k, *v, *hcat, *ao, *x, *xa, *xn2, *xlast;
  float* scores;                 /* per thread: max_ctx */
  int n_threads;
  float* inv_freq;               /* head_dim / 2 */
  double* moe_ms;
  long* moe_calls;
  double cpu_ms;
  int moe_uploaded;
  /* expert parallelism (mh_ep_setup / mh_ep_connect): device staging of the
     MoE block's input and residual rows, and the stream of moe_ffn_ep */
  int ep_on, ep_cap;
  float *d_xn, *d_xo;
  cudaStream_t ep_stream;
};

static _Thread_local char g_err[512];   /* per calling thread */

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

const char* mh_last_error(void) { return g_err; }

static double now_ms(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

static float* own(MhModel* m, size_t n) {
  float* p = (float*)malloc(sizeof(float) * (n ? n : 1));
  if (!p) return NULL;
  if (m->n_owned == m->cap_owned) {
    int nc = m->cap_owned ? 2 * m->cap_owned : 64;
    float** o = (float**)realloc(m->owned, sizeof(float*) * (size_t)nc);
    if (!o) { free(p); return NULL; }
    m->owned = o;
    m->cap_owned = nc;
  }
  m->owned[m->n_owned++] = p;
  return p;
}

/* ---- CPU arithmetic (bit-compatible with the reference) ------------------- */

/* AVX2 form of the same chains: 16 outputs per pass, two 8-lane
   accumulators. Each 8x8 tile of weights (8 rows x 8 consecutive k) is
   transposed in registers so that lane j of column i holds w[n0+j][k+i];
   the lanes then add a[k+i]*w in k order, one separately rounded multiply
   and add at a time, exactly the scalar chain of each output. */
__attribute__((target("avx2"))) static inline void transpose8(__m256 r[8]) {
  const __m256 t0 = _mm256_unpacklo_ps(r[0], r[1]), t1 = _mm256_unpackhi_ps(r[0], r[1]);
  const __m256 t2 = _mm256_unpacklo_ps(r[2], r[3]), t3 = _mm256_unpackhi_ps(r[2], r[3]);
  const __m256 t4 = _mm256_unpacklo_ps(r[4], r[5]), t5 = _mm256_unpackhi_ps(r[4], r[5]);
  const __m256 t6 = _mm256_unpacklo_ps(r[6], r[7]), t7 = _mm256_unpackhi_ps(r[6], r[7]);
  const __m256 s0 = _mm256_shuffle_ps(t0, t2, 0x44), s1 = _mm256_shuffle_ps(t0, t2, 0xEE);
  const __m256 s2 = _mm256_shuffle_ps(t1, t3, 0x44), s3 = _mm256_shuffle_ps(t1, t3, 0xEE);
  const __m256 s4 = _mm256_shuffle_ps(t4, t6, 0x44), s5 = _mm256_shuffle_ps(t4, t6, 0xEE);
  const __m256 s6 = _mm256_shuffle_ps(t5, t7, 0x44), s7 = _mm256_shuffle_ps(t5, t7, 0xEE);
  r[0] = _mm256_permute2f128_ps(s0, s4, 0x20); r[1] = _mm256_permute2f128_ps(s1, s5, 0x20);
  r[2] = _mm256_permute2f128_ps(s2, s6, 0x20); r[3] = _mm256_permute2f128_ps(s3, s7, 0x20);
  r[4] = _mm256_permute2f128_ps(s0, s4, 0x31); r[5] = _mm256_permute2f128_ps(s1, s5, 0x31);
  r[6] = _mm256_permute2f128_ps(s2, s6, 0x31); r[7] = _mm256_permute2f128_ps(s3, s7, 0x31);
}

/* c[j] = chain(a . w[j]) for the 16 rows w + j*ldw, j = 0..15 */
__attribute__((target("avx2"))) static void dot16_avx2(const float* a, const float* w, size_t ldw, float* c,
                                                       int K) {
  __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
  const int K8 = K & ~7;
  for (int k = 0; k < K8; k += 8) {
    __m256 r[8], q[8];
    for (int j = 0; j < 8; ++j) {
      r[j] = _mm256_loadu_ps(w + (size_t)j * ldw + k);
      q[j] = _mm256_loadu_ps(w + (size_t)(j + 8) * ldw + k);
    }
    transpose8(r);
    transpose8(q);
    for (int i = 0; i < 8; ++i) {
      const __m256 av = _mm256_set1_ps(a[k + i]);
      acc0 = _mm256_add_ps(acc0, _mm256_mul_ps(av, r[i]));
      acc1 = _mm256_add_ps(acc1, _mm256_mul_ps(av, q[i]));
    }
  }
  float acc[16];
  _mm256_storeu_ps(acc, acc0);
  _mm256_storeu_ps(acc + 8, acc1);
  for (int k = K8; k < K; ++k)
    for (int j = 0; j < 16; ++j) acc[j] += a[k] * w[(size_t)j * ldw + k];
  memcpy(c, acc, sizeof(acc));
}

/* Rows m0..m0+nm-1 (nm <= 64) of A against the 16 rows w + j*ldw: each 16x8
   weight tile is transposed once and applied to every row; the per-row
   accumulators live in acc[nm][16] between tiles. Same chains as
   dot16_avx2, row by row. */
__attribute__((target("avx2"))) static void dot16_rows_avx2(const float* A, size_t lda, int nm, const float* w,
                                                            size_t ldw, float* C, size_t ldc, int K) {
  float acc[64 * 16] __attribute__((aligned(32)));
  memset(acc, 0, sizeof(float) * 16 * (size_t)nm);
  const int K8 = K & ~7;
  for (int k = 0; k < K8; k += 8) {
    __m256 r[8], q[8];
    for (int j = 0; j < 8; ++j) {
      r[j] = _mm256_loadu_ps(w + (size_t)j * ldw + k);
      q[j] = _mm256_loadu_ps(w + (size_t)(j + 8) * ldw + k);
    }
    transpose8(r);
    transpose8(q);
    for (int m = 0; m < nm; ++m) {
      const float* a = A + (size_t)m * lda + k;
      __m256 acc0 = _mm256_load_ps(acc + 16 * m), acc1 = _mm256_load_ps(acc + 16 * m + 8);
      for (int i = 0; i < 8; ++i) {
        const __m256 av = _mm256_set1_ps(a[i]);
        acc0 = _mm256_add_ps(acc0, _mm256_mul_ps(av, r[i]));
        acc1 = _mm256_add_ps(acc1, _mm256_mul_ps(av, q[i]));
      }
      _mm256_store_ps(acc + 16 * m, acc0);
      _mm256_store_ps(acc + 16 * m + 8, acc1);
    }
  }
  for (int m = 0; m < nm; ++m) {
    float* am = acc + 16 * m;
    const float* a = A + (size_t)m * lda;
    for (int k = K8; k < K; ++k)
      for (int j = 0; j < 16; ++j) am[j] += a[k] * w[(size_t)j * ldw + k];
    memcpy(C + (size_t)m * ldc, am, sizeof(float) * 16);
  }
}

/* out[d] += p * v[d] for d < n: independent lanes, one rounded multiply and
   add each, in the caller's key order */
__attribute__((target("avx2"))) static void axpy_avx2(float p, const float* v, float* out, int n) {
  const __m256 pv = _mm256_set1_ps(p);
  int d = 0;
  for (; d + 8 <= n; d += 8)
    _mm256_storeu_ps(out + d, _mm256_add_ps(_mm256_loadu_ps(out + d), _mm256_mul_ps(pv, _mm256_loadu_ps(v + d))));
  for (; d < n; ++d) out[d] += p * v[d];
}

/* MOE_HOST_SCALAR=1 keeps the portable path (for tests and comparisons) */
static int use_avx2(void) {
  static int v = -1;
  if (v < 0) {
    __builtin_cpu_init();
    const char* e = getenv("MOE_HOST_SCALAR");
    v = !(e && atoi(e)) && __builtin_cpu_supports("avx2");
  }
  return v;
}

/* C[M][N] = A[M][K] . W[N][K]^T, each output one sequential chain. */
static void mm_f32(const float* A, const float* W, float* C, int M, int N, int K) {
  if (use_avx2() && N >= 16) {
    const int nb = N / 16;
#pragma omp parallel for schedule(static)
    for (int b = 0; b < nb; ++b) {
      if (M == 1) {
        dot16_avx2(A, W + (size_t)16 * b * K, (size_t)K, C + 16 * b, K);
        continue;
      }
      for (int m0 = 0; m0 < M; m0 += 64)
        dot16_rows_avx2(A + (size_t)m0 * K, (size_t)K, M - m0 < 64 ? M - m0 : 64, W + (size_t)16 * b * K,
                        (size_t)K, C + (size_t)m0 * N + 16 * b, (size_t)N, K);
    }
    const int n_done = nb * 16;
    for (int m = 0; m < M; ++m)
      for (int n = n_done; n < N; ++n) {
        const float* a = A + (size_t)m * K;
        const float* w = W + (size_t)n * K;
        float acc = 0.f;
        for (int k = 0; k < K; ++k) acc += a[k] * w[k];
        C[(size_t)m * N + n] = acc;
      }
    return;
  }
  const int nb = (N + 3) / 4;
#pragma omp parallel for schedule(static)
  for (int b = 0; b < nb; ++b) {
    const int n0 = 4 * b;
    for (int m = 0; m < M; ++m) {
      const float* a = A + (size_t)m * K;
      float* c = C + (size_t)m * N;
      if (n0 + 4 <= N) {
        const float* w0 = W + (size_t)n0 * K;
        const float* w1 = w0 + K;
        const float* w2 = w1 + K;
        const float* w3 = w2 + K;
        float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
        for (int k = 0; k < K; ++k) {
          const float av = a[k];
          c0 += av * w0[k];
          c1 += av * w1[k];
          c2 += av * w2[k];
          c3 += av * w3[k];
        }
        c[n0] = c0; c[n0 + 1] = c1; c[n0 + 2] = c2; c[n0 + 3] = c3;
      } else {
        for (int n = n0; n < N; ++n) {
          const float* w = W + (size_t)n * K;
          float acc = 0.f;
          for (int k = 0; k < K; ++k) acc += a[k] * w[k];
          c[n] = acc;
        }
      }
    }
  }
}

static void rmsnorm_rows(const float* x, const float* w, int R, int D, float eps, float* y) {
#pragma omp parallel for schedule(static) if (R > 1)
  for (int r = 0; r < R; ++r) {
    const float* xt = x + (size_t)r * D;
    float* yt = y + (size_t)r * D;
    float msq = 0.0f;
    for (int i = 0; i < D; ++i) msq += xt[i] * xt[i];
    msq /= (float)D;
    const float inv = 1.0f / sqrtf(msq + eps);
    for (int i = 0; i < D; ++i) yt[i] = xt[i] * inv * (w ? w[i] : 1.0f);
  }
}

static void head_norm(float* v, const float* w, int hd, float eps) {
  float msq = 0.f;
  for (int d = 0; d < hd; ++d) { const float z = v[d]; msq += z * z; }
  const float inv = 1.0f / sqrtf(msq / (float)hd + eps);
  for (int d = 0; d < hd; ++d) v[d] = (v[d] * inv) * w[d];
}

static void rope_row(float* h, const float* inv_freq, int d2, float p) {
  for (int i = 0; i < d2; ++i) {
    const float ang = p * inv_freq[i];
    const float c = cosf(ang), s = sinf(ang);
    const float e = h[i], o = h[i + d2];
    h[i] = e * c - o * s;
    h[i + d2] = o * c + e * s;
  }
}

/* ---- model ------------------------------------------------------------------ */

MhModel* mh_create(const MhConfig* cfg, int batch, int max_ctx, int moe_layer_base) {
  if (!cfg || batch < 1 || max_ctx < 1 || cfg->n_layers < 1 || cfg->d_model < 1 || cfg->head_dim < 2 ||
      (cfg->head_dim & 1) || cfg->n_q < 1 || cfg->n_kv < 1 || cfg->n_q % cfg->n_kv || cfg->vocab_size < 1) {
    fail(MOE_ERR_INVALID, "mh_create: bad config or sizes");
    return NULL;
  }
  MhModel* m = (MhModel*)calloc(1, sizeof(MhModel));
  if (!m) { fail(MOE_ERR_NOMEM, "mh_create: out of host memory"); return NULL; }
  m->c = *cfg;
  m->batch = batch;
  m->max_ctx = max_ctx;
  m->moe_base = moe_layer_base;
  m->Dq = cfg->n_q * cfg->head_dim;
  m->Dkv = cfg->n_kv * cfg->head_dim;
  m->layers = (Layer*)calloc((size_t)cfg->n_layers, sizeof(Layer));
  const size_t kv = (size_t)cfg->n_layers * batch * max_ctx * m->Dkv;
  m->kc = (float*)malloc(sizeof(float) * kv);
  m->vc = (float*)malloc(sizeof(float) * kv);
  m->n_threads = omp_get_max_threads();
  m->scores = (float*)malloc(sizeof(float) * (size_t)m->n_threads * max_ctx);
  m->inv_freq = (float*)malloc(sizeof(float) * (size_t)(cfg->head_dim / 2));
  m->moe_ms = (double*)calloc((size_t)cfg->n_layers, sizeof(double));
  m->moe_calls = (long*)calloc((size_t)cfg->n_layers, sizeof(long));
  if (!m->layers || !m->kc || !m->vc || !m->scores || !m->inv_freq || !m->moe_ms || !m->moe_calls) {
    mh_free(m);
    fail(MOE_ERR_NOMEM, "mh_create: out of host memory (KV cache %zu bytes)", 2 * sizeof(float) * kv);
    return NULL;
  }
  for (int i = 0; i < cfg->head_dim / 2; ++i) {
    const float exponent = -2.0f * (float)i / (float)cfg->head_dim;
    m->inv_freq[i] = powf(cfg->rope_theta, exponent);
  }
  return m;
}

/* The MoE block's input and residual rows (xn2, x, xa: x and xa swap every
   layer) are page-locked and mapped, so each moe_ffn call copies xn2 in and
   updates the residual in place through its mapped address, with no copy
   out; plain malloc if page-locked memory is refused (the call then copies). */
static float* rows_alloc(MhModel* m, size_t bytes) {
  void* p = NULL;
  if (m->pinned_rows && cudaHostAlloc(&p, bytes, cudaHostAllocMapped) == cudaSuccess) return (float*)p;
  cudaGetLastError();
  m->pinned_rows = 0;
  return (float*)malloc(bytes);
}

static void rows_free(MhModel* m, float* p) {
  if (!p) return;
  if (cudaFreeHost(p) != cudaSuccess) { cudaGetLastError(); free(p); }
  (void)m;
}

static void free_scratch(MhModel* m) {
  float* s[] = {m->xn1, m->q, m->k, m->v, m->hcat, m->ao, m->xlast};
  for (size_t i = 0; i < sizeof(s) / sizeof(s[0]); ++i) free(s[i]);
  rows_free(m, m->x); rows_free(m, m->xa); rows_free(m, m->xn2);
  m->xn1 = m->q = m->k = m->v = m->hcat = m->ao = m->x = m->xa = m->xn2 = m->xlast = NULL;
  m->cap_rows = 0;
}

void mh_free(MhModel* m) {
  if (!m) return;
  if (m->d_xn) cudaFree(m->d_xn);
  if (m->d_xo) cudaFree(m->d_xo);
  if (m->ep_stream) cudaStreamDestroy(m->ep_stream);
  if (m->moe_uploaded)
    for (int l = 0; l < m->c.n_layers; ++l) moe_cuda_free_layer(m->moe_base + l);
  for (int i = 0; i < m->n_owned; ++i) free(m->owned[i]);
  free(m->owned);
  free_scratch(m);
  free(m->layers); free(m->kc); free(m->vc); free(m->scores); free(m->inv_freq);
  free(m->moe_ms); free(m->moe_calls);
  free(m);
}

static int ensure_rows(MhModel* m, int R) {
  if (R <= m->cap_rows) return MOE_OK;
  free_scratch(m);
  const size_t D = (size_t)m->c.d_model;
  m->xn1 = (float*)malloc(sizeof(float) * R * D);
  m->q = (float*)malloc(sizeof(float) * R * (size_t)m->Dq);
  m->k = (float*)malloc(sizeof(float) * R * (size_t)m->Dkv);
  m->v = (float*)malloc(sizeof(float) * R * (size_t)m->Dkv);
  m->hcat = (float*)malloc(sizeof(float) * R * (size_t)m->Dq);
  m->ao = (float*)malloc(sizeof(float) * R * D);
  m->pinned_rows = 1;
  m->x = rows_alloc(m, sizeof(float) * R * D);
  m->xa = rows_alloc(m, sizeof(float) * R * D);
  m->xn2 = rows_alloc(m, sizeof(float) * R * D);
  m->xlast = (float*)malloc(sizeof(float) * (size_t)m->batch * D);
  if (!m->xn1 || !m->q || !m->k || !m->v || !m->hcat || !m->ao || !m->x || !m->xa || !m->xn2 || !m->xlast) {
    free_scratch(m);
    return fail(MOE_ERR_NOMEM, "step scratch for %d rows", R);
  }
  m->cap_rows = R;
  return MOE_OK;
}

int mh_set_globals(MhModel* m, const float* tok_emb, const float* final_norm_w, const float* lm_head) {
  if (!m || !tok_emb || !final_norm_w) return fail(MOE_ERR_INVALID, "mh_set_globals: NULL argument");
  m->tok_emb = tok_emb;
  m->final_norm_w = final_norm_w;
  m->lm_head = lm_head;
  return MOE_OK;
}

int mh_set_layer(MhModel* m, int layer, const MhLayerWeights* w) {
  if (!m || !w || layer < 0 || layer >= m->c.n_layers) return fail(MOE_ERR_INVALID, "mh_set_layer: bad layer");
  if (!w->Wq || !w->Wk || !w->Wv || !w->Wo || !w->rms1_w || !w->rms2_w)
    return fail(MOE_ERR_INVALID, "mh_set_layer: layer %d lacks a projection or norm", layer);
  m->layers[layer].w = *w;
  return MOE_OK;
}

int mh_pos(const MhModel* m) { return m ? m->pos : 0; }
void mh_reset(MhModel* m) { if (m) m->pos = 0; }

int mh_advance(MhModel* m, int T) {
  if (!m || T < 0 || m->pos + T > m->max_ctx) return fail(MOE_ERR_INVALID, "mh_advance: past max_ctx");
  m->pos += T;
  return MOE_OK;
}

int mh_embed(MhModel* m, const int* ids, int T, float* x) {
  if (!m || !ids || !x || T < 1) return fail(MOE_ERR_INVALID, "mh_embed: bad argument");
  if (!m->tok_emb) return fail(MOE_ERR_NOT_INIT, "mh_embed: no embedding set");
  const int D = m->c.d_model;
  for (int r = 0; r < m->batch * T; ++r) {
    const int id = ids[r];
    if (id < 0 || id >= m->c.vocab_size) return fail(MOE_ERR_INVALID, "token id %d out of range", id);
    memcpy(x + (size_t)r * D, m->tok_emb + (size_t)id * D, sizeof(float) * (size_t)D);
  }
  return MOE_OK;
}

static float* kv_row(const MhModel* m, float* base, int layer, int b, int p) {
  return base + (((size_t)layer * m->batch + b) * m->max_ctx + p) * m->Dkv;
}

int mh_attention(MhModel* m, int layer, const float* x, int T, float* x_after, float* x_norm2) {
  if (!m || layer < 0 || layer >= m->c.n_layers || !x || !x_after || !x_norm2 || T < 1)
    return fail(MOE_ERR_INVALID, "mh_attention: bad argument");
  if (m->pos + T > m->max_ctx) return fail(MOE_ERR_INVALID, "mh_attention: position %d + %d > max_ctx %d",
                                          m->pos, T, m->max_ctx);
  const MhLayerWeights* w = &m->layers[layer].w;
  if (!w->Wq) return fail(MOE_ERR_NOT_INIT, "mh_attention: layer %d has no weights", layer);
  const int R = m->batch * T, D = m->c.d_model, Dq = m->Dq, Dkv = m->Dkv, hd = m->c.head_dim;
  const int nq = m->c.n_q, nkv = m->c.n_kv, group = nq / nkv, d2 = hd / 2;
  const float eps = m->c.rms_eps;
  int rc = ensure_rows(m, R);
  if (rc) return rc;
  const double t0 = now_ms();

  rmsnorm_rows(x, w->rms1_w, R, D, eps, m->xn1);
  mm_f32(m->xn1, w->Wq, m->q, R, Dq, D);
  mm_f32(m->xn1, w->Wk, m->k, R, Dkv, D);
  mm_f32(m->xn1, w->Wv, m->v, R, Dkv, D);
  for (int r = 0; r < R; ++r) {
    if (w->bq) for (int i = 0; i < Dq; ++i) m->q[(size_t)r * Dq + i] += w->bq[i];
    if (w->bk) for (int i = 0; i < Dkv; ++i) m->k[(size_t)r * Dkv + i] += w->bk[i];
    if (w->bv) for (int i = 0; i < Dkv; ++i) m->v[(size_t)r * Dkv + i] += w->bv[i];
  }
#pragma omp parallel for schedule(static)
  for (int r = 0; r < R; ++r) {
    const float p = (float)(m->pos + r % T);
    float* qr = m->q + (size_t)r * Dq;
    float* kr = m->k + (size_t)r * Dkv;
    if (w->q_norm) for (int h = 0; h < nq; ++h) head_norm(qr + (size_t)h * hd, w->q_norm, hd, eps);
    if (w->k_norm) for (int h = 0; h < nkv; ++h) head_norm(kr + (size_t)h * hd, w->k_norm, hd, eps);
    for (int h = 0; h < nq; ++h) rope_row(qr + (size_t)h * hd, m->inv_freq, d2, p);
    for (int h = 0; h < nkv; ++h) rope_row(kr + (size_t)h * hd, m->inv_freq, d2, p);
    const int b = r / T, t = r % T;
    memcpy(kv_row(m, m->kc, layer, b, m->pos + t), kr, sizeof(float) * (size_t)Dkv);
    memcpy(kv_row(m, m->vc, layer, b, m->pos + t), m->v + (size_t)r * Dkv, sizeof(float) * (size_t)Dkv);
  }

  /* one task per (sequence, query head, new token); one score row per thread */
  const float scale = 1.0f / sqrtf((float)hd);
  const int avx = use_avx2();
  const int tasks = m->batch * nq * T;
  const int nth = omp_get_max_threads();
  if (nth > m->n_threads) {
    float* sc = (float*)realloc(m->scores, sizeof(float) * (size_t)nth * m->max_ctx);
    if (!sc) return fail(MOE_ERR_NOMEM, "attention score rows for %d threads", nth);
    m->scores = sc;
    m->n_threads = nth;
  }
#pragma omp parallel for schedule(dynamic, 1) num_threads(nth)
  for (int task = 0; task < tasks; ++task) {
    const int t = task % T, h = (task / T) % nq, b = task / (T * nq);
    const int kvh = h / group;
    const int P = m->pos + t;                           /* keys 0..P */
    float* S = m->scores + (size_t)omp_get_thread_num() * m->max_ctx;
    const float* qv = m->q + ((size_t)b * T + t) * Dq + (size_t)h * hd;
    /* scores: keys are rows of stride Dkv, so 16 keys at a time take the
       matmul's transposed-lane chains; the rest one chain each */
    const int tk16 = avx ? (P + 1) & ~15 : 0;
    for (int tk = 0; tk < tk16; tk += 16) {
      dot16_avx2(qv, kv_row(m, m->kc, layer, b, tk) + (size_t)kvh * hd, (size_t)Dkv, S + tk, hd);
      for (int j = 0; j < 16; ++j) S[tk + j] = S[tk + j] * scale;
    }
    for (int tk = tk16; tk <= P; ++tk) {
      const float* kv = kv_row(m, m->kc, layer, b, tk) + (size_t)kvh * hd;
      float dot = 0.f;
      for (int d = 0; d < hd; ++d) dot += qv[d] * kv[d];
      S[tk] = dot * scale;
    }
    float mx = S[0];
    for (int i = 1; i <= P; ++i) if (S[i] > mx) mx = S[i];
    float ssum = 0.f;
    for (int i = 0; i <= P; ++i) { const float e = expf(S[i] - mx); S[i] = e; ssum += e; }
    const float inv = 1.f / (ssum + 1e-9f);
    for (int i = 0; i <= P; ++i) S[i] *= inv;
    float* out = m->hcat + ((size_t)b * T + t) * Dq + (size_t)h * hd;
    for (int d = 0; d < hd; ++d) out[d] = 0.f;
    for (int tk = 0; tk <= P; ++tk) {
      const float* vv = kv_row(m, m->vc, layer, b, tk) + (size_t)kvh * hd;
      const float pr = S[tk];
      if (avx) axpy_avx2(pr, vv, out, hd);
      else for (int d = 0; d < hd; ++d) out[d] += pr * vv[d];
    }
  }

  mm_f32(m->hcat, w->Wo, m->ao, R, D, Dq);
  if (w->bo) for (int r = 0; r < R; ++r) for (int i = 0; i < D; ++i) m->ao[(size_t)r * D + i] += w->bo[i];
  for (size_t i = 0; i < (size_t)R * D; ++i) x_after[i] = x[i] + m->ao[i];
  rmsnorm_rows(x_after, w->rms2_w, R, D, eps, x_norm2);
  m->cpu_ms += now_ms() - t0;
  return MOE_OK;
}

/* Expert-parallel MoE block of R rows: moe_ffn_ep over the rows in chunks of
   at most ep_cap (every rank has the same R, so the chunks line up across
   the ranks), through device staging, then the status check. */
static int moe_ep_rows(MhModel* m, int layer, const float* x_norm2, float* x_after, int R) {
  const size_t D = (size_t)m->c.d_model;
  for (int r0 = 0; r0 < R; r0 += m->ep_cap) {
    const int n = R - r0 < m->ep_cap ? R - r0 : m->ep_cap;
    const size_t bytes = sizeof(float) * (size_t)n * D;
    if (cudaMemcpyAsync(m->d_xn, x_norm2 + (size_t)r0 * D, bytes, cudaMemcpyHostToDevice, m->ep_stream) ||
        cudaMemcpyAsync(m->d_xo, x_after + (size_t)r0 * D, bytes, cudaMemcpyHostToDevice, m->ep_stream))
      return fail(MOE_ERR_CUDA, "mh_moe: copy to the device failed");
    int rc = moe_ffn_ep(m->moe_base + layer, m->d_xn, n, m->d_xo, m->ep_stream);
    if (rc) return fail(rc, "moe_ffn_ep (layer %d): %s", layer, moe_cuda_last_error());
    if (cudaMemcpyAsync(x_after + (size_t)r0 * D, m->d_xo, bytes, cudaMemcpyDeviceToHost, m->ep_stream) ||
        cudaStreamSynchronize(m->ep_stream))
      return fail(MOE_ERR_CUDA, "mh_moe: copy from the device failed");
    if ((rc = moe_cuda_check_status())) return fail(rc, "moe_ffn_ep (layer %d): %s", layer, moe_cuda_last_error());
  }
  return MOE_OK;
}

int mh_ep_setup(MhModel* m, int max_rows_per_call, void* handle_out) {
  if (!m || max_rows_per_call < 1 || !handle_out) return fail(MOE_ERR_INVALID, "mh_ep_setup: bad argument");
  const size_t bytes = sizeof(float) * (size_t)max_rows_per_call * m->c.d_model;
  if (!m->d_xn && (cudaMalloc((void**)&m->d_xn, bytes) || cudaMalloc((void**)&m->d_xo, bytes) ||
                   cudaStreamCreateWithFlags(&m->ep_stream, cudaStreamNonBlocking)))
    return fail(MOE_ERR_NOMEM, "mh_ep_setup: device staging of %d rows", max_rows_per_call);
  const int rc = moe_cuda_ep_setup(max_rows_per_call, m->c.d_model, 8, handle_out);
  if (rc) return fail(rc, "moe_cuda_ep_setup: %s", moe_cuda_last_error());
  m->ep_cap = max_rows_per_call;
  return MOE_OK;
}

int mh_ep_connect(MhModel* m, const void* handles) {
  if (!m || !handles || !m->ep_cap) return fail(MOE_ERR_INVALID, "mh_ep_connect: call mh_ep_setup first");
  const int rc = moe_cuda_ep_connect(handles);
  if (rc) return fail(rc, "moe_cuda_ep_connect: %s", moe_cuda_last_error());
  m->ep_on = 1;
  return MOE_OK;
}

int mh_moe(MhModel* m, int layer, const float* x_norm2, float* x_after, int T) {
  if (!m || layer < 0 || layer >= m->c.n_layers) return fail(MOE_ERR_INVALID, "mh_moe: bad layer");
  const double t0 = now_ms();
  if (m->ep_on) {
    const int rc = moe_ep_rows(m, layer, x_norm2, x_after, m->batch * T);
    if (rc) return rc;
    m->moe_ms[layer] += now_ms() - t0;
    m->moe_calls[layer] += 1;
    return MOE_OK;
  }
  const int rc = moe_ffn(m->moe_base + layer, x_norm2, x_after, m->batch * T, NULL, NULL,
                         MOE_FFN_HOST_PTRS, NULL);
  if (rc) return fail(rc, "moe_ffn (layer %d): %s", layer, moe_cuda_last_error());
  m->moe_ms[layer] += now_ms() - t0;
  m->moe_calls[layer] += 1;
  return MOE_OK;
}

int mh_head(MhModel* m, const float* x, int T, float* logits) {
  if (!m || !x || !logits || T < 1) return fail(MOE_ERR_INVALID, "mh_head: bad argument");
  if (!m->final_norm_w) return fail(MOE_ERR_NOT_INIT, "mh_head: no final norm set");
  int rc = ensure_rows(m, m->batch * T);
  if (rc) return rc;
  const double t0 = now_ms();
  const int D = m->c.d_model;
  for (int b = 0; b < m->batch; ++b)
    memcpy(m->xn1 + (size_t)b * D, x + ((size_t)b * T + T - 1) * D, sizeof(float) * (size_t)D);
  rmsnorm_rows(m->xn1, m->final_norm_w, m->batch, D, m->c.rms_eps, m->xlast);
  mm_f32(m->xlast, m->lm_head ? m->lm_head : m->tok_emb, logits, m->batch, m->c.vocab_size, D);
  m->cpu_ms += now_ms() - t0;
  return MOE_OK;
}

int mh_step(MhModel* m, const int* ids, int T, float* logits) {
  if (!m || !ids || !logits || T < 1) return fail(MOE_ERR_INVALID, "mh_step: bad argument");
  int rc = ensure_rows(m, m->batch * T);
  if (rc) return rc;
  if ((rc = mh_embed(m, ids, T, m->x))) return rc;
  for (int l = 0; l < m->c.n_layers; ++l) {
    if ((rc = mh_attention(m, l, m->x, T, m->xa, m->xn2))) return rc;
    if ((rc = mh_moe(m, l, m->xn2, m->xa, T))) return rc;
    float* t = m->x; m->x = m->xa; m->xa = t;      /* x <- x_after + moe */
  }
  if ((rc = mh_head(m, m->x, T, logits))) return rc;
  return mh_advance(m, T);
}

/* softmax_rows (test_model_trace.c:260-272) on one row, then the first
   maximum (:723-731) */
static int softmax_argmax(float* row, int n) {
  float maxv = row[0];
  for (int c = 1; c < n; ++c) if (row[c] > maxv) maxv = row[c];
  float sum = 0.f;
  for (int c = 0; c < n; ++c) { const float e = expf(row[c] - maxv); row[c] = e; sum += e; }
  const float inv = 1.0f / (sum + 1e-9f);
  for (int c = 0; c < n; ++c) row[c] *= inv;
  int best = 0;
  float bv = row[0];
  for (int c = 1; c < n; ++c) if (row[c] > bv) { bv = row[c]; best = c; }
  return best;
}

int mh_pick_greedy(const MhModel* m, float* logits, int* ids) {
  if (!m || !logits || !ids) return fail(MOE_ERR_INVALID, "mh_pick_greedy: NULL argument");
  for (int b = 0; b < m->batch; ++b) ids[b] = softmax_argmax(logits + (size_t)b * m->c.vocab_size, m->c.vocab_size);
  return MOE_OK;
}

int mh_generate(MhModel* m, const int* prompts, int prompt_len, int steps, int* out) {
  if (!m || !prompts || !out || prompt_len < 1 || steps < 1) return fail(MOE_ERR_INVALID, "mh_generate: bad argument");
  if (prompt_len + steps - 1 > m->max_ctx) return fail(MOE_ERR_INVALID, "mh_generate: exceeds max_ctx");
  const int B = m->batch, V = m->c.vocab_size;
  float* logits = (float*)malloc(sizeof(float) * (size_t)B * V);
  int* ids = (int*)malloc(sizeof(int) * (size_t)B);
  if (!logits || !ids) { free(logits); free(ids); return fail(MOE_ERR_NOMEM, "mh_generate: host memory"); }
  mh_reset(m);
  int rc = mh_step(m, prompts, prompt_len, logits);
  for (int s = 0; !rc && s < steps; ++s) {
    mh_pick_greedy(m, logits, ids);
    for (int b = 0; b < B; ++b) out[(size_t)b * steps + s] = ids[b];
    if (s + 1 < steps) rc = mh_step(m, ids, 1, logits);
  }
  free(logits); free(ids);
  return rc;
}

int mh_timing(const MhModel* m, double* moe_ms, long* moe_calls, double* cpu_ms) {
  if (!m) return fail(MOE_ERR_INVALID, "mh_timing: NULL model");
  for (int l = 0; l < m->c.n_layers; ++l) {
    if (moe_ms) moe_ms[l] = m->moe_ms[l];
    if (moe_calls) moe_calls[l] = m->moe_calls[l];
  }
  if (cpu_ms) *cpu_ms = m->cpu_ms;
  return MOE_OK;
}

void mh_timing_reset(MhModel* m) {
  if (!m) return;
  memset(m->moe_ms, 0, sizeof(double) * (size_t)m->c.n_layers);
  memset(m->moe_calls, 0, sizeof(long) * (size_t)m->c.n_layers);
  m->cpu_ms = 0;
}

/* ---- weights from a .bin file (model.h:107-210) ---------------------------- */

static const char* find_any(MoeBin* b, char* buf, size_t n, const char* f1, const char* f2, int L) {
  snprintf(buf, n, f1, L);
  if (moe_bin_find(b, buf, NULL, NULL, NULL, NULL) == MOE_OK) return buf;
  if (!f2) return NULL;
  snprintf(buf, n, f2, L);
  if (moe_bin_find(b, buf, NULL, NULL, NULL, NULL) == MOE_OK) return buf;
  return NULL;
}

int mh_config_from_bin(const char* path, MhConfig* cfg) {
  if (!cfg) return fail(MOE_ERR_INVALID, "mh_config_from_bin: NULL cfg");
  MoeBin* b = moe_bin_open(path);
  if (!b) return fail(MOE_ERR_INVALID, "%s", moe_cuda_last_error());
  int rc = MOE_OK;
  int sq[8], sk[8], se[8], sn[8], nd;
  if (moe_bin_find(b, "model.layers.0.self_attn.q_proj.weight", NULL, &nd, sq, NULL) ||
      moe_bin_find(b, "model.layers.0.self_attn.k_proj.weight", NULL, &nd, sk, NULL) ||
      moe_bin_find(b, "model.embed_tokens.weight", NULL, &nd, se, NULL)) {
    rc = fail(MOE_ERR_INVALID, "%s", moe_cuda_last_error());
    goto out;
  }
  memset(cfg, 0, sizeof(*cfg));
  cfg->d_model = sq[1];
  cfg->head_dim = moe_bin_find(b, "model.layers.0.self_attn.q_norm.weight", NULL, &nd, sn, NULL) == MOE_OK
                      ? sn[0] : sq[0] / 32;
  cfg->n_q = sq[0] / cfg->head_dim;
  cfg->n_kv = sk[0] / cfg->head_dim;
  cfg->vocab_size = se[0];
  for (;;) {
    char k[128];
    snprintf(k, sizeof(k), "model.layers.%d.self_attn.q_proj.weight", cfg->n_layers);
    if (moe_bin_find(b, k, NULL, NULL, NULL, NULL) != MOE_OK) break;
    cfg->n_layers++;
  }
  int E, D, F, dt, hb;
  if ((rc = moe_bin_layer_info_h(b, 0, &E, &D, &F, &dt, &hb))) {
    rc = fail(rc, "%s", moe_cuda_last_error());
    goto out;
  }
  cfg->n_experts = E;
  cfg->d_ff = F;
  cfg->rope_theta = 10000000.f;   /* model.h:119-120 */
  cfg->rms_eps = 1e-6f;
out:
  moe_bin_close(b);
  return rc;
}

static const float* read_f32(MhModel* m, MoeBin* b, const char* name, size_t n, int* rc) {
  int dt, nd, shape[8];
  size_t nb;
  if (*rc) return NULL;
  if (moe_bin_find(b, name, &dt, &nd, shape, &nb) || dt != 0 || nb != sizeof(float) * n) {
    *rc = fail(MOE_ERR_INVALID, "%s: missing, not f32 or not %zu elements", name, n);
    return NULL;
  }
  float* p = own(m, n);
  if (!p) { *rc = fail(MOE_ERR_NOMEM, "host memory for %s", name); return NULL; }
  if (moe_bin_read(b, name, p, nb)) { *rc = fail(MOE_ERR_INVALID, "%s", moe_cuda_last_error()); return NULL; }
  return p;
}

static const float* read_opt_f32(MhModel* m, MoeBin* b, const char* name, size_t n, int* rc) {
  int dt;
  size_t nb;
  if (*rc || moe_bin_find(b, name, &dt, NULL, NULL, &nb) != MOE_OK || dt != 0) return NULL;
  return read_f32(m, b, name, n, rc);
}

int mh_load_bin(MhModel* m, const char* path) {
  if (!m) return fail(MOE_ERR_INVALID, "mh_load_bin: NULL model");
  MhConfig fc;
  int rc = mh_config_from_bin(path, &fc);
  if (rc) return rc;
  const MhConfig* c = &m->c;
  if (fc.d_model != c->d_model || fc.n_layers < c->n_layers || fc.head_dim != c->head_dim || fc.n_q != c->n_q ||
      fc.n_kv != c->n_kv || fc.vocab_size != c->vocab_size || fc.n_experts != c->n_experts || fc.d_ff != c->d_ff)
    return fail(MOE_ERR_INVALID, "%s: shapes differ from the model's config", path);
  MoeBin* b = moe_bin_open(path);
  if (!b) return fail(MOE_ERR_INVALID, "%s", moe_cuda_last_error());
  const size_t D = (size_t)c->d_model, V = (size_t)c->vocab_size, hd = (size_t)c->head_dim;
  char k[160];
  m->tok_emb = read_f32(m, b, "model.embed_tokens.weight", V * D, &rc);
  const char* nn = find_any(b, k, sizeof(k), "model.norm.weight", "model.final_layernorm.weight", 0);
  m->final_norm_w = nn ? read_f32(m, b, nn, D, &rc) : NULL;
  if (!rc && !nn) rc = fail(MOE_ERR_INVALID, "%s: no final norm", path);
  m->lm_head = read_opt_f32(m, b, "lm_head.weight", V * D, &rc);
  for (int L = 0; L < c->n_layers && !rc; ++L) {
    MhLayerWeights w;
    memset(&w, 0, sizeof(w));
#define RD(field, fmt, n) do { snprintf(k, sizeof(k), fmt, L); w.field = read_f32(m, b, k, (n), &rc); } while (0)
#define RO(field, fmt, n) do { snprintf(k, sizeof(k), fmt, L); w.field = read_opt_f32(m, b, k, (n), &rc); } while (0)
    RD(Wq, "model.layers.%d.self_attn.q_proj.weight", (size_t)m->Dq * D);
    RD(Wk, "model.layers.%d.self_attn.k_proj.weight", (size_t)m->Dkv * D);
    RD(Wv, "model.layers.%d.self_attn.v_proj.weight", (size_t)m->Dkv * D);
    RD(Wo, "model.layers.%d.self_attn.o_proj.weight", D * (size_t)m->Dq);
    RO(bq, "model.layers.%d.self_attn.q_proj.bias", (size_t)m->Dq);
    RO(bk, "model.layers.%d.self_attn.k_proj.bias", (size_t)m->Dkv);
    RO(bv, "model.layers.%d.self_attn.v_proj.bias", (size_t)m->Dkv);
    RO(bo, "model.layers.%d.self_attn.o_proj.bias", D);
    RO(q_norm, "model.layers.%d.self_attn.q_norm.weight", hd);
    RO(k_norm, "model.layers.%d.self_attn.k_norm.weight", hd);
#undef RD
#undef RO
    const char* n1 = find_any(b, k, sizeof(k), "model.layers.%d.input_layernorm.weight", "model.layers.%d.rms_1.weight", L);
    w.rms1_w = n1 ? read_f32(m, b, n1, D, &rc) : NULL;
    const char* n2 = find_any(b, k, sizeof(k), "model.layers.%d.post_attention_layernorm.weight",
                              "model.layers.%d.rms_2.weight", L);
    w.rms2_w = n2 ? read_f32(m, b, n2, D, &rc) : NULL;
    if (!rc && (!n1 || !n2)) rc = fail(MOE_ERR_INVALID, "%s: layer %d lacks its norms", path, L);
    if (!rc) rc = mh_set_layer(m, L, &w);
    if (!rc) {
      m->moe_uploaded = 1;
      if ((rc = moe_cuda_load_bin_layer_h(b, L, m->moe_base + L))) rc = fail(rc, "%s", moe_cuda_last_error());
    }
  }
  moe_bin_close(b);
  return rc;
}

/* ---- random-init weights ------------------------------------------------------ */

static uint64_t stream_seed(uint64_t seed, uint64_t layer, uint64_t tid) {
  return seed * 1000003ull + layer * 1009ull + tid;
}

#define CUDA_OK(call, what)                                                                      \
  do {                                                                                           \
    cudaError_t e_ = (call);                                                                     \
    if (e_ != cudaSuccess) { rc = fail(MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e_)); goto out; } \
  } while (0)

int mh_synth(MhModel* m, uint64_t seed, int expert_dtype, float std) {
  if (!m || (expert_dtype != MOE_DTYPE_Q8 && expert_dtype != MOE_DTYPE_Q4))
    return fail(MOE_ERR_INVALID, "mh_synth: bad argument");
  const MhConfig* c = &m->c;
  const size_t D = (size_t)c->d_model, V = (size_t)c->vocab_size, F = (size_t)c->d_ff, E = (size_t)c->n_experts;
  const size_t hd = (size_t)c->head_dim;
  const int q8 = expert_dtype == MOE_DTYPE_Q8;
  int rc = MOE_OK;
  float* tmp = NULL;               /* device fp32 staging (largest tensor) */
  unsigned char* dq = NULL;        /* device quantised experts of one layer */
  float* ds = NULL;
  QuantizedWeight* W = (QuantizedWeight*)calloc(3 * E, sizeof(QuantizedWeight));
  size_t big = V * D;
  if ((size_t)m->Dq * D > big) big = (size_t)m->Dq * D;
  if (F * D > big) big = F * D;
  if (E * D > big) big = E * D;
  if (!W) return fail(MOE_ERR_NOMEM, "mh_synth: host memory");
  const size_t qrow_gu = q8 ? D : D / 2, qrow_d = q8 ? F : F / 2;
  const size_t qbytes = E * (2 * F * qrow_gu + D * qrow_d);
  CUDA_OK(cudaMalloc((void**)&tmp, sizeof(float) * big), "device staging");
  CUDA_OK(cudaMalloc((void**)&dq, qbytes), "device expert staging");
  CUDA_OK(cudaMalloc((void**)&ds, sizeof(float) * E * (2 * F + D)), "device scale staging");

  /* host fp32 tensor `tid` of layer `layer`, n elements */
#define HOST_T(dst, layer, tid, n)                                                                  \
  do {                                                                                              \
    float* p_ = own(m, (n));                                                                        \
    if (!p_) { rc = fail(MOE_ERR_NOMEM, "mh_synth: host memory"); goto out; }                      \
    if ((rc = moe_synth_normal_dev(stream_seed(seed, (layer), (tid)), 0, (n), std, tmp, NULL))) {   \
      rc = fail(rc, "%s", moe_cuda_last_error()); goto out;                                         \
    }                                                                                               \
    CUDA_OK(cudaMemcpy(p_, tmp, sizeof(float) * (n), cudaMemcpyDeviceToHost), "copy to host");      \
    (dst) = p_;                                                                                     \
  } while (0)

  {
    const float *emb, *fn, *head;
    HOST_T(emb, 65535, 0, V * D);
    HOST_T(fn, 65535, 1, D);
    HOST_T(head, 65535, 2, V * D);
    mh_set_globals(m, emb, fn, head);
  }
  for (int L = 0; L < c->n_layers; ++L) {
    MhLayerWeights w;
    memset(&w, 0, sizeof(w));
    HOST_T(w.Wq, L, 100000, (size_t)m->Dq * D);
    HOST_T(w.Wk, L, 100001, (size_t)m->Dkv * D);
    HOST_T(w.Wv, L, 100002, (size_t)m->Dkv * D);
    HOST_T(w.Wo, L, 100003, D * (size_t)m->Dq);
    HOST_T(w.q_norm, L, 100004, hd);
    HOST_T(w.k_norm, L, 100005, hd);
    HOST_T(w.rms1_w, L, 100006, D);
    HOST_T(w.rms2_w, L, 100007, D);
    if ((rc = mh_set_layer(m, L, &w))) goto out;
    /* experts: drawn and quantised on the device, then made resident */
    unsigned char* qp = dq;
    float* sp = ds;
    for (size_t e = 0; e < E; ++e) {
      for (int j = 0; j < 3; ++j) {
        const size_t rows = j < 2 ? F : D, cols = j < 2 ? D : F, qr = j < 2 ? qrow_gu : qrow_d;
        if (!(rc = moe_synth_normal_dev(stream_seed(seed, L, 2 + 3 * e + j), 0, rows * cols, std, tmp, NULL)))
          rc = q8 ? moe_quantize_rowwise_q8_dev(tmp, (int)rows, (int)cols, (int8_t*)qp, sp, NULL)
                  : moe_quantize_rowwise_q4_dev(tmp, (int)rows, (int)cols, (uint8_t*)qp, sp, NULL);
        if (rc) {
          rc = fail(rc, "%s", moe_cuda_last_error());
          goto out;
        }
        QuantizedWeight* qw = &W[j * E + e];
        qw->q = (const int8_t*)qp; qw->s = sp;
        qw->rows = (int)rows; qw->cols = (int)cols; qw->dtype = expert_dtype;
        qp += rows * qr;
        sp += rows;
      }
    }
    if ((rc = moe_synth_normal_dev(stream_seed(seed, L, 0), 0, E * D, std, tmp, NULL))) {
      rc = fail(rc, "%s", moe_cuda_last_error());
      goto out;
    }
    m->moe_uploaded = 1;
    if ((rc = moe_cuda_upload_layer_dev(m->moe_base + L, W, W + E, W + 2 * E, tmp, NULL, (int)E))) {
      rc = fail(rc, "%s", moe_cuda_last_error());
      goto out;
    }
  }
#undef HOST_T
out:
  cudaDeviceSynchronize();
  cudaFree(tmp);
  cudaFree(dq);
  cudaFree(ds);
  free(W);
  return rc;
}

int mh_fill_kv(MhModel* m, int ctx, uint64_t seed, float std) {
  if (!m || ctx < 0 || ctx > m->max_ctx) return fail(MOE_ERR_INVALID, "mh_fill_kv: bad context");
  int rc = MOE_OK;
  const size_t row = (size_t)ctx * m->Dkv;           /* one (layer, sequence) block */
  float* tmp = NULL;
  if (row == 0) { m->pos = ctx; return MOE_OK; }
  CUDA_OK(cudaMalloc((void**)&tmp, sizeof(float) * row), "device staging");
  for (int l = 0; l < m->c.n_layers; ++l)
    for (int b = 0; b < m->batch; ++b)
      for (int kv = 0; kv < 2; ++kv) {
        const uint64_t blk = ((uint64_t)l * m->batch + b) * 2 + kv;
        if ((rc = moe_synth_normal_dev(stream_seed(seed, 65534, blk), 0, row, std, tmp, NULL))) {
          rc = fail(rc, "%s", moe_cuda_last_error());
          goto out;
        }
        CUDA_OK(cudaMemcpy(kv_row(m, kv ? m->vc : m->kc, l, b, 0), tmp, sizeof(float) * row,
                           cudaMemcpyDeviceToHost), "copy to host");
      }
  m->pos = ctx;
out:
  cudaFree(tmp);
  return rc;
}

/* ---- model.c call surface (include/moe_model.h) ------------------------------
 * layer_forward_f32 / model_forward_f32 with model.c's parameter lists
 * (model.c:38-58, :192-198). The CPU parts restate model.c:59-131 and
 * :199-252 with the helpers above; the MoE block (:133-187) runs on the GPU:
 * the fp32 experts resident (moe_cuda_upload_layer_f32), moe_ffn with
 * MOE_FFN_SEQ_RESIDUAL (p*y added straight into x, slot by slot, :188) and,
 * when the caller passes a routing, MOE_FFN_GIVEN_TOPK. */
#include <pthread.h>
#include "../../include/moe_model.h"

typedef struct {
  const float* router_w;
  const float* wg0;
  int E, D, F, topk, id;
} F32Layer;

static pthread_mutex_t g_f32_mu = PTHREAD_MUTEX_INITIALIZER;
static F32Layer* g_f32;
static int g_nf32, g_cap_f32;
#define MOE_MODEL_LAYER_BASE 0x70000000

static void model_die(const char* who, const char* msg) {
  fprintf(stderr, "libmoe_host: %s failed: %s\n", who, msg);
  abort();
}

/* The resident copy of a layer's fp32 experts: uploaded on first use. */
static int f32_layer_id(const float* router_w, const float* router_b, const float** Wg, const float** Wu,
                        const float** Wd, int E, int D, int F, int topk) {
  pthread_mutex_lock(&g_f32_mu);
  int id = -1;
  for (int i = 0; i < g_nf32; ++i) {
    const F32Layer* l = &g_f32[i];
    if (l->router_w == router_w && l->wg0 == Wg[0] && l->E == E && l->D == D && l->F == F && l->topk == topk) {
      id = l->id;
      break;
    }
  }
  if (id < 0) {
    moe_cuda_init(0, 1, 0, NULL);  /* no-op (or a harmless refusal) when already initialised */
    if (g_nf32 == g_cap_f32) {
      const int nc = g_cap_f32 ? 2 * g_cap_f32 : 16;
      F32Layer* nl = (F32Layer*)realloc(g_f32, sizeof(F32Layer) * (size_t)nc);
      if (!nl) { pthread_mutex_unlock(&g_f32_mu); model_die("layer_forward_f32", "out of host memory"); }
      g_f32 = nl;
      g_cap_f32 = nc;
    }
    id = MOE_MODEL_LAYER_BASE + g_nf32;
    const int rc = moe_cuda_upload_layer_f32(id, (const float* const*)Wg, (const float* const*)Wu,
                                             (const float* const*)Wd, router_w, router_b, E, D, F, topk);
    if (rc) { pthread_mutex_unlock(&g_f32_mu); model_die("layer_forward_f32 (upload)", moe_cuda_last_error()); }
    F32Layer l = {router_w, Wg[0], E, D, F, topk, id};
    g_f32[g_nf32++] = l;
  }
  pthread_mutex_unlock(&g_f32_mu);
  return id;
}

void moe_model_release(void) {
  pthread_mutex_lock(&g_f32_mu);
  for (int i = 0; i < g_nf32; ++i) moe_cuda_free_layer(g_f32[i].id);
  free(g_f32);
  g_f32 = NULL;
  g_nf32 = g_cap_f32 = 0;
  pthread_mutex_unlock(&g_f32_mu);
}

/* model.c:59-131: norm1, attention over all T positions from 0, residual,
   norm2. Causal masking only removes keys that add exactly 0. */
static void model_attention(float* x, int T, int D, const float* rms1_w, float rms1_eps, const float* Wq,
                            const float* bq, const float* Wk, const float* bk, const float* Wv, const float* bv,
                            const float* Wo, const float* bo, const float* qn, const float* kn, int n_q, int n_kv,
                            int dh, int causal, float rope_theta, const float* rms2_w, float rms2_eps,
                            float* scratch, float* x_norm2) {
  const int Dq = n_q * dh, Dkv = n_kv * dh, d2 = dh / 2, group = n_q / n_kv;
  const float scale = 1.0f / sqrtf((float)dh);
  float* Q = scratch;
  float* K = Q + (size_t)T * Dq;
  float* V = K + (size_t)T * Dkv;
  float* S = V + (size_t)T * Dkv;                 /* [T][T] */
  float* Hcat = S + (size_t)T * T;
  float* x_norm1 = Hcat + (size_t)T * Dq;
  float* attn_out = x_norm1 + (size_t)T * D;
  rmsnorm_rows(x, rms1_w, T, D, rms1_eps, x_norm1);
  mm_f32(x_norm1, Wq, Q, T, Dq, D);
  mm_f32(x_norm1, Wk, K, T, Dkv, D);
  mm_f32(x_norm1, Wv, V, T, Dkv, D);
  for (int t = 0; t < T; ++t) {
    if (bq) for (int i = 0; i < Dq; ++i) Q[(size_t)t * Dq + i] += bq[i];
    if (bk) for (int i = 0; i < Dkv; ++i) K[(size_t)t * Dkv + i] += bk[i];
    if (bv) for (int i = 0; i < Dkv; ++i) V[(size_t)t * Dkv + i] += bv[i];
  }
  float* inv_freq = (float*)malloc(sizeof(float) * (size_t)(d2 > 0 ? d2 : 1));
  if (!inv_freq) model_die("layer_forward_f32", "out of host memory");
  for (int i = 0; i < d2; ++i) inv_freq[i] = powf(rope_theta, -2.0f * (float)i / (float)dh);
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    float* Qt = Q + (size_t)t * Dq;
    float* Kt = K + (size_t)t * Dkv;
    if (qn && kn) {                                 /* model.c:81-88, eps fixed at 1e-6 */
      for (int h = 0; h < n_q; ++h) head_norm(Qt + (size_t)h * dh, qn, dh, 1e-6f);
      for (int h = 0; h < n_kv; ++h) head_norm(Kt + (size_t)h * dh, kn, dh, 1e-6f);
    }
    for (int h = 0; h < n_q; ++h) rope_row(Qt + (size_t)h * dh, inv_freq, d2, (float)t);
    for (int h = 0; h < n_kv; ++h) rope_row(Kt + (size_t)h * dh, inv_freq, d2, (float)t);
  }
  free(inv_freq);
  /* one (head, query) per task; S row tq of the task's own head is private
     to the task because tasks of one head never share a query row */
  float* Sh = (float*)malloc(sizeof(float) * (size_t)n_q * T * T);
  if (!Sh) model_die("layer_forward_f32", "out of host memory (attention scores)");
#pragma omp parallel for schedule(dynamic, 4)
  for (int task = 0; task < n_q * T; ++task) {
    const int h = task / T, tq = task % T, kvh = h / group;
    const int last = causal ? tq : T - 1;            /* later keys are -inf: exp gives 0 */
    const float* qv = Q + (size_t)tq * Dq + (size_t)h * dh;
    float* Sout = Sh + ((size_t)h * T + tq) * T;
    for (int tk = 0; tk <= last; ++tk) {
      const float* kv = K + (size_t)tk * Dkv + (size_t)kvh * dh;
      float dot = 0.f;
      for (int d = 0; d < dh; ++d) dot += qv[d] * kv[d];
      Sout[tk] = dot * scale;
    }
    float m = Sout[0];
    for (int i = 1; i <= last; ++i) if (Sout[i] > m) m = Sout[i];
    float s = 0.f;
    for (int i = 0; i <= last; ++i) { const float z = expf(Sout[i] - m); Sout[i] = z; s += z; }
    const float inv = 1.f / (s + 1e-9f);
    for (int i = 0; i <= last; ++i) Sout[i] *= inv;
    float* out = Hcat + (size_t)tq * Dq + (size_t)h * dh;
    for (int d = 0; d < dh; ++d) out[d] = 0.f;
    for (int tk = 0; tk <= last; ++tk) {
      const float* vv = V + (size_t)tk * Dkv + (size_t)kvh * dh;
      const float p = Sout[tk];
      for (int d = 0; d < dh; ++d) out[d] += p * vv[d];
    }
  }
  /* the reference's S buffer holds the last head's probabilities on return */
  if (n_q > 0) memcpy(S, Sh + (size_t)(n_q - 1) * T * T, sizeof(float) * (size_t)T * T);
  free(Sh);
  mm_f32(Hcat, Wo, attn_out, T, D, Dq);
  if (bo) for (int t = 0; t < T; ++t) for (int i = 0; i < D; ++i) attn_out[(size_t)t * D + i] += bo[i];
  for (size_t i = 0; i < (size_t)T * D; ++i) x[i] = x[i] + attn_out[i];
  rmsnorm_rows(x, rms2_w, T, D, rms2_eps, x_norm2);
}

void layer_forward_f32(float* x, int T, int D, const float* rms1_w, float rms1_eps, const float* Wq,
                       const float* bq, const float* Wk, const float* bk, const float* Wv, const float* bv,
                       const float* Wo, const float* bo, const float* qn, const float* kn, int n_q, int n_kv,
                       int head_dim, int causal, float rope_theta, const float* rms2_w, float rms2_eps,
                       const float* router_w, const float* router_b, const float** Wg, const float** bg,
                       const float** Wu, const float** bu, const float** Wd, const float** bd, int n_experts,
                       int topk, int d_ff, float* scratch_attn, float* scratch_moe, int* reuse_topk_idx,
                       float* reuse_topk_p) {
  (void)bg; (void)bu; (void)bd; (void)scratch_moe;   /* model.c reads neither */
  if (T <= 0) return;
  if (!x || D <= 0 || !Wq || !Wk || !Wv || !Wo || !router_w || n_q < 1 || n_kv < 1 || n_q % n_kv ||
      head_dim < 2 || (head_dim & 1) || !scratch_attn)
    model_die("layer_forward_f32", "bad argument");
  if (!Wg || !Wu || !Wd || !Wg[0])
    model_die("layer_forward_f32", "model.c's layer takes fp32 experts (Wg/Wu/Wd, model.c:172-187)");
  const int id = f32_layer_id(router_w, router_b, Wg, Wu, Wd, n_experts, D, d_ff, topk);
  float* x_norm2 = (float*)malloc(sizeof(float) * (size_t)T * D);
  if (!x_norm2) model_die("layer_forward_f32", "out of host memory");
  model_attention(x, T, D, rms1_w, rms1_eps, Wq, bq, Wk, bk, Wv, bv, Wo, bo, qn, kn, n_q, n_kv, head_dim, causal,
                  rope_theta, rms2_w, rms2_eps, scratch_attn, x_norm2);
  const int given = reuse_topk_idx && reuse_topk_p;
  const int rc = moe_ffn(id, x_norm2, x, T, given ? reuse_topk_idx : NULL, given ? reuse_topk_p : NULL,
                         MOE_FFN_HOST_PTRS | MOE_FFN_SEQ_RESIDUAL | (given ? MOE_FFN_GIVEN_TOPK : 0), NULL);
  free(x_norm2);
  if (rc) model_die("layer_forward_f32 (moe_ffn)", moe_cuda_last_error());
}

void model_forward_f32(const int* ids, int T, const QwenConfig* cfg, const QwenWeights* w, int apply_softmax,
                       float* out_logits) {
  if (T <= 0) return;
  if (!ids || !cfg || !w || !out_logits || !w->tok_emb || !w->final_norm_w || !w->layers)
    model_die("model_forward_f32", "bad argument");
  const int D = cfg->d_model, V = cfg->vocab_size, L = cfg->n_layers, dh = cfg->head_dim;
  const int Dq = cfg->n_q * dh, Dkv = cfg->n_kv * dh;
  const size_t attn_f = (size_t)T * (Dq + 2 * Dkv) + (size_t)T * T + (size_t)T * Dq + 2ull * T * D;
  float* scratch = (float*)malloc(sizeof(float) * attn_f);
  float* x = (float*)malloc(sizeof(float) * (size_t)T * D);
  float* x_final = (float*)malloc(sizeof(float) * (size_t)T * D);
  if (!scratch || !x || !x_final) model_die("model_forward_f32", "out of host memory");
  for (int t = 0; t < T; ++t) {
    if (ids[t] < 0 || ids[t] >= V) model_die("model_forward_f32", "token id out of range");
    memcpy(x + (size_t)t * D, w->tok_emb + (size_t)ids[t] * D, sizeof(float) * (size_t)D);
  }
  for (int l = 0; l < L; ++l) {
    const QwenLayerWeights* lw = &w->layers[l];
    layer_forward_f32(x, T, D, lw->rms1_w, 1e-6f, lw->Wq, lw->bq, lw->Wk, lw->bk, lw->Wv, lw->bv, lw->Wo,
                      lw->bo, lw->q_norm, lw->k_norm, cfg->n_q, cfg->n_kv, dh, cfg->causal, cfg->rope_theta,
                      lw->rms2_w, 1e-6f, lw->router_w, lw->router_b, lw->Wg, lw->bg, lw->Wu, lw->bu, lw->Wd,
                      lw->bd, cfg->n_experts, cfg->top_k, cfg->d_ff, scratch, NULL, NULL, NULL);
  }
  rmsnorm_rows(x, w->final_norm_w, T, D, 1e-6f, x_final);
  mm_f32(x_final, w->lm_head ? w->lm_head : w->tok_emb, out_logits, T, V, D);
  if (apply_softmax) {                              /* softmax_rows, model.c:10-28 */
    for (int r = 0; r < T; ++r) {
      float* row = out_logits + (size_t)r * V;
      float maxv = row[0];
      for (int c = 1; c < V; ++c) if (row[c] > maxv) maxv = row[c];
      float sum = 0.0f;
      for (int c = 0; c < V; ++c) { row[c] = expf(row[c] - maxv); sum += row[c]; }
      const float inv = 1.0f / (sum + 1e-9f);
      for (int c = 0; c < V; ++c) row[c] *= inv;
    }
  }
  free(x_final);
  free(x);
  free(scratch);
}
