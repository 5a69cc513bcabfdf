/*
 * ref_shim.c — call-in shim for the REFERENCE's own compiled code.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product). Built by
 * oracle/Makefile, only where the reference sources are present, into
 * oracle/_ref/libmoe_ref.so together with the reference's unmodified
 * kernels.c, io.c and utils.c, all with the reference's own flags
 * (gcc -O2 -Wall -DDEBUG -DBENCH, Makefile:2-3). No reference source is
 * copied into this repository: the #include below reads test_model_trace.c
 * where it lies (REF_DIR on the include path).
 *
 * test_model_trace.c's layer_forward_f32 (:433-521) is static, so this file
 * is compiled in the same translation unit and exposes one entry,
 * ref_moe_layer(), that runs the reference's real layer_forward_f32 with an
 * attention block whose weights are all zero (1 query head, 1 KV head,
 * head_dim 2). Attention then adds exactly 0 (Wo = 0), so x_after == x, and
 * the MoE block that follows (:463-517) is the reference's code verbatim,
 * including matmul_adaptive -> matmul_f32_q8/_q4 from kernels.c. The MoE
 * input x_norm2 = rmsnorm(x) (rms2_w = NULL, eps 1e-6) is read back from
 * the caller-owned scratch buffer, where layer_forward_f32 leaves it.
 */
#define main moe_ref_trace_main_unused
#include "test_model_trace.c"
#undef main

/* Clear the reference profiler's table so its atexit dump prints nothing
 * (PROFILING is hard-wired on, test_model_trace.c:64). */
static void ref_prof_clear(void) {
  memset(__prof_tab, 0, sizeof(__prof_tab));
}

/*
 * x_in: [T][D]   layer input x (MoE sees x_norm2 = rmsnorm(x))
 * x_out: [T][D]  x after the layer (= x + moe_out)
 * x_norm2_out: [T][D]  the MoE block's input, as the reference computed it
 * logits_out: [T][E]   router logits (+bias) from the reference
 * idx_out/p_out: [T][topk] the reference's topk_desc + top-k softmax of each
 *   token's logits (recomputed per token with the reference's own topk_desc;
 *   layer_forward_f32 keeps only the last token's in tmp_idx/tmp_val)
 * Expert arrays as orc_moe_block (contiguous per projection).
 */
int ref_moe_layer(const float* x_in, float* x_out, float* x_norm2_out,
                  float* logits_out, int* idx_out, float* p_out,
                  int T, int D, int E, int topk, int F,
                  const float* router_w, const float* router_b, int dtype,
                  const void* gq, const float* gs, const void* uq,
                  const float* us, const void* dq, const float* ds) {
  if (dtype != 2 && dtype != 3) return -1;
  const int hd = 2, nq = 1, nkv = 1;
  const size_t gu_row = dtype == 2 ? (size_t)D : (size_t)D / 2;
  const size_t d_row = dtype == 2 ? (size_t)F : (size_t)F / 2;

  float* Wq = (float*)calloc((size_t)nq * hd * D, sizeof(float));
  float* Wk = (float*)calloc((size_t)nkv * hd * D, sizeof(float));
  float* Wv = (float*)calloc((size_t)nkv * hd * D, sizeof(float));
  float* Wo = (float*)calloc((size_t)D * nq * hd, sizeof(float));
  QuantizedWeight* g = (QuantizedWeight*)calloc((size_t)E, sizeof(QuantizedWeight));
  QuantizedWeight* u = (QuantizedWeight*)calloc((size_t)E, sizeof(QuantizedWeight));
  QuantizedWeight* d = (QuantizedWeight*)calloc((size_t)E, sizeof(QuantizedWeight));
  for (int e = 0; e < E; ++e) {
    g[e].q = (const int8_t*)gq + (size_t)e * F * gu_row; g[e].s = gs + (size_t)e * F;
    u[e].q = (const int8_t*)uq + (size_t)e * F * gu_row; u[e].s = us + (size_t)e * F;
    d[e].q = (const int8_t*)dq + (size_t)e * D * d_row;  d[e].s = ds + (size_t)e * D;
    g[e].rows = u[e].rows = F; g[e].cols = u[e].cols = D;
    d[e].rows = D; d[e].cols = F;
    g[e].dtype = u[e].dtype = d[e].dtype = dtype;
  }
  QwenLayerWeights lw;
  memset(&lw, 0, sizeof(lw));
  lw.Wq = Wq; lw.Wk = Wk; lw.Wv = Wv; lw.Wo = Wo;
  lw.router_w = router_w; lw.router_b = router_b;
  lw.Wg_q = g; lw.Wu_q = u; lw.Wd_q = d;
  lw.experts_quantized = 1;

  /* scratch sizes exactly as model_forward_f32 allocates them (:537-540) */
  const int Dq = nq * hd, Dkv = nkv * hd;
  size_t attn_f = (size_t)T * (Dq + 2 * Dkv) + (size_t)T * T + (size_t)T * Dq;
  size_t temps_f = 4ull * (size_t)T * D;
  float* scratch_attn = (float*)malloc(sizeof(float) * (attn_f + temps_f));
  float* scratch_moe = (float*)malloc(sizeof(float) * ((size_t)T * E + (size_t)T * D));
  int* tmp_idx = (int*)malloc(sizeof(int) * (size_t)topk);
  float* tmp_val = (float*)malloc(sizeof(float) * (size_t)topk);
  memcpy(x_out, x_in, sizeof(float) * (size_t)T * D);

  layer_forward_f32(x_out, T, D, &lw, nq, nkv, hd, /*causal=*/1,
                    /*rope_theta=*/10000000.f, /*rms_eps=*/1e-6f,
                    E, topk, F, scratch_attn, scratch_moe, tmp_idx, tmp_val);

  /* x_norm2 sits after x_norm1, attn_out, x_after (test_model_trace.c:443-446) */
  const float* x_norm2 = scratch_attn + attn_f + 3ull * (size_t)T * D;
  if (x_norm2_out) memcpy(x_norm2_out, x_norm2, sizeof(float) * (size_t)T * D);
  if (logits_out) memcpy(logits_out, scratch_moe, sizeof(float) * (size_t)T * E);
  for (int t = 0; t < T && (idx_out || p_out); ++t) {
    topk_desc(scratch_moe + (size_t)t * E, E, topk, tmp_idx, tmp_val);
    float maxv = tmp_val[0];
    for (int i = 1; i < topk; ++i) if (tmp_val[i] > maxv) maxv = tmp_val[i];
    float sum = 0.f;
    for (int i = 0; i < topk; ++i) { tmp_val[i] = expf(tmp_val[i] - maxv); sum += tmp_val[i]; }
    float inv = 1.0f / (sum + 1e-9f);
    for (int i = 0; i < topk; ++i) tmp_val[i] *= inv;
    if (idx_out) memcpy(idx_out + (size_t)t * topk, tmp_idx, sizeof(int) * (size_t)topk);
    if (p_out) memcpy(p_out + (size_t)t * topk, tmp_val, sizeof(float) * (size_t)topk);
  }

  free(Wq); free(Wk); free(Wv); free(Wo); free(g); free(u); free(d);
  free(scratch_attn); free(scratch_moe); free(tmp_idx); free(tmp_val);
  ref_prof_clear();
  return 0;
}

/* The reference's matmul_adaptive (kernels.c:149-181), called with a
 * QuantizedWeight built from plain arguments. dtype 0 = fp32 (W_q NULL). */
int ref_matmul(const float* A, const void* Wq, const float* Ws, const float* Wf,
               float* C, int M, int N, int K, int dtype) {
  QuantizedWeight w;
  w.q = (const int8_t*)Wq; w.s = Ws; w.rows = N; w.cols = K; w.dtype = dtype;
  matmul_adaptive(A, Wf, dtype == 0 ? NULL : &w, C, M, N, K);
  return 0;
}

/*
 * The reference's whole model_forward_f32 (test_model_trace.c:526-596) on
 * caller-provided weights: logits of the last of T tokens.
 *   attn: n_layers x 12 pointers (Wq, bq, Wk, bk, Wv, bv, Wo, bo, q_norm,
 *         k_norm, rms1_w, rms2_w; biases and q/k norms may be NULL)
 *   router: n_layers x 2 (router_w, router_b or NULL)
 *   experts: n_layers x 6 (gq, gs, uq, us, dq, ds, contiguous per projection
 *            as in ref_moe_layer)
 * top_k 8, causal (model.h:159-161).
 */
int ref_model_forward(const int* ids, int T, int D, int n_layers, int head_dim, int n_q, int n_kv,
                      int F, int E, int V, float rope_theta, float rms_eps,
                      const float* tok_emb, const float* final_norm_w, const float* lm_head,
                      const float* const* attn, const float* const* router, int dtype,
                      const void* const* experts, float* out_last) {
  if (dtype != 2 && dtype != 3) return -1;
  QwenConfig cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.d_model = D; cfg.n_layers = n_layers; cfg.head_dim = head_dim; cfg.n_q = n_q; cfg.n_kv = n_kv;
  cfg.d_ff = F; cfg.n_experts = E; cfg.top_k = 8; cfg.vocab_size = V; cfg.causal = 1;
  cfg.rope_theta = rope_theta; cfg.rms_eps = rms_eps;
  QwenWeights w;
  memset(&w, 0, sizeof(w));
  w.tok_emb = tok_emb; w.final_norm_w = final_norm_w; w.lm_head = lm_head;
  w.layers = (QwenLayerWeights*)calloc((size_t)n_layers, sizeof(QwenLayerWeights));
  QuantizedWeight* qw = (QuantizedWeight*)calloc((size_t)n_layers * 3 * E, sizeof(QuantizedWeight));
  const size_t gu_row = dtype == 2 ? (size_t)D : (size_t)D / 2;
  const size_t d_row = dtype == 2 ? (size_t)F : (size_t)F / 2;
  for (int l = 0; l < n_layers; ++l) {
    QwenLayerWeights* lw = &w.layers[l];
    const float* const* a = attn + 12 * l;
    lw->Wq = a[0]; lw->bq = a[1]; lw->Wk = a[2]; lw->bk = a[3]; lw->Wv = a[4]; lw->bv = a[5];
    lw->Wo = a[6]; lw->bo = a[7]; lw->q_norm = a[8]; lw->k_norm = a[9]; lw->rms1_w = a[10]; lw->rms2_w = a[11];
    lw->router_w = router[2 * l]; lw->router_b = router[2 * l + 1];
    const void* const* x = experts + 6 * l;
    QuantizedWeight* g = qw + (size_t)l * 3 * E;
    QuantizedWeight* u = g + E;
    QuantizedWeight* d = u + E;
    for (int e = 0; e < E; ++e) {
      g[e].q = (const int8_t*)x[0] + (size_t)e * F * gu_row; g[e].s = (const float*)x[1] + (size_t)e * F;
      u[e].q = (const int8_t*)x[2] + (size_t)e * F * gu_row; u[e].s = (const float*)x[3] + (size_t)e * F;
      d[e].q = (const int8_t*)x[4] + (size_t)e * D * d_row;  d[e].s = (const float*)x[5] + (size_t)e * D;
      g[e].rows = u[e].rows = F; g[e].cols = u[e].cols = D;
      d[e].rows = D; d[e].cols = F;
      g[e].dtype = u[e].dtype = d[e].dtype = dtype;
    }
    lw->Wg_q = g; lw->Wu_q = u; lw->Wd_q = d;
    lw->experts_quantized = 1;
  }
  model_forward_f32(ids, T, &cfg, &w, /*apply_softmax=*/0, out_last);
  free(w.layers);
  free(qw);
  ref_prof_clear();
  return 0;
}

/*
 * The reference's model.c, compiled from its source in this translation
 * unit. model.c does not build on its own as shipped: model.h uses fprintf
 * without <stdio.h>, and the helpers it calls (matmul_f32, silu_f32,
 * rmsnorm_forward_f32, rope_apply_inplace_f32_gqa) are the static ones of
 * test_model_trace.c included above. Its two exported names collide with
 * test_model_trace.c's statics, so they are renamed on the way in, as is its
 * own static softmax_rows. Its text is otherwise compiled unchanged.
 *
 * model_forward_f32 (model.c:212-214) sizes scratch_attn for the attention
 * buffers only, and layer_forward_f32 then writes x_norm2 (T*D floats) and
 * the router logits (T*E floats) past its end (model.c:130, :134). To run it
 * without corrupting the heap, model.c's malloc calls get 16 MiB of slack.
 */
#include <alloca.h>   /* model.c calls alloca without declaring it */
static void* refmc_malloc(size_t n) { return malloc(n + ((size_t)16 << 20)); }
#define layer_forward_f32 refmc_layer_forward_f32
#define model_forward_f32 refmc_model_forward_f32
#define softmax_rows refmc_softmax_rows
#define malloc(n) refmc_malloc(n)
#include "model.c"
#undef malloc
#undef softmax_rows
#undef model_forward_f32
#undef layer_forward_f32

/*
 * model.c's model_forward_f32 on caller-provided fp32 weights: logits of all
 * T rows [T][V] (softmaxed if apply_softmax).
 *   attn: n_layers x 12 pointers as ref_model_forward
 *   router: n_layers x 2 (router_w, router_b or NULL)
 *   experts: n_layers x 3 pointers (gate [E][F][D], up [E][F][D], down
 *            [E][D][F], fp32, contiguous per projection)
 */
int ref_mc_model_forward(const int* ids, int T, int D, int n_layers, int head_dim, int n_q, int n_kv,
                         int F, int E, int top_k, int V, float rope_theta, int causal,
                         const float* tok_emb, const float* final_norm_w, const float* lm_head,
                         const float* const* attn, const float* const* router, const float* const* experts,
                         int apply_softmax, float* out_logits) {
  QwenConfig cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.d_model = D; cfg.n_layers = n_layers; cfg.head_dim = head_dim; cfg.n_q = n_q; cfg.n_kv = n_kv;
  cfg.d_ff = F; cfg.n_experts = E; cfg.top_k = top_k; cfg.vocab_size = V; cfg.causal = causal;
  cfg.rope_theta = rope_theta; cfg.rms_eps = 1e-6f;
  QwenWeights w;
  memset(&w, 0, sizeof(w));
  w.tok_emb = tok_emb; w.final_norm_w = final_norm_w; w.lm_head = lm_head;
  w.layers = (QwenLayerWeights*)calloc((size_t)n_layers, sizeof(QwenLayerWeights));
  const float** ptrs = (const float**)calloc((size_t)n_layers * 3 * E, sizeof(float*));
  for (int l = 0; l < n_layers; ++l) {
    QwenLayerWeights* lw = &w.layers[l];
    const float* const* a = attn + 12 * l;
    lw->Wq = a[0]; lw->bq = a[1]; lw->Wk = a[2]; lw->bk = a[3]; lw->Wv = a[4]; lw->bv = a[5];
    lw->Wo = a[6]; lw->bo = a[7]; lw->q_norm = a[8]; lw->k_norm = a[9]; lw->rms1_w = a[10]; lw->rms2_w = a[11];
    lw->router_w = router[2 * l]; lw->router_b = router[2 * l + 1];
    const float** g = ptrs + (size_t)l * 3 * E;
    const float** u = g + E;
    const float** d = u + E;
    for (int e = 0; e < E; ++e) {
      g[e] = experts[3 * l] + (size_t)e * F * D;
      u[e] = experts[3 * l + 1] + (size_t)e * F * D;
      d[e] = experts[3 * l + 2] + (size_t)e * D * F;
    }
    lw->Wg = g; lw->Wu = u; lw->Wd = d;
  }
  refmc_model_forward_f32(ids, T, &cfg, &w, apply_softmax, out_logits);
  free(ptrs);
  free(w.layers);
  ref_prof_clear();
  return 0;
}

/* model.c's layer_forward_f32 on one layer (fp32 experts as above), x in
 * place; reuse_idx/reuse_p as model.c's reuse_topk_idx/p (both NULL: the
 * layer computes its own routing). */
int ref_mc_layer_forward(float* x, int T, int D, const float* const* a, float rms1_eps, float rms2_eps,
                         int n_q, int n_kv, int head_dim, int causal, float rope_theta,
                         const float* router_w, const float* router_b, const float* gate, const float* up,
                         const float* down, int E, int top_k, int F, int* reuse_idx, float* reuse_p) {
  const int Dq = n_q * head_dim, Dkv = n_kv * head_dim;
  float* scratch_attn = (float*)calloc((size_t)T * (Dq + 2 * Dkv) + (size_t)T * T + (size_t)T * Dq +
                                       4ull * T * D + (size_t)T * E, sizeof(float));
  float* scratch_moe = (float*)calloc(2ull * T * F, sizeof(float));
  const float** ptrs = (const float**)calloc((size_t)3 * E, sizeof(float*));
  for (int e = 0; e < E; ++e) {
    ptrs[e] = gate + (size_t)e * F * D;
    ptrs[E + e] = up + (size_t)e * F * D;
    ptrs[2 * E + e] = down + (size_t)e * D * F;
  }
  refmc_layer_forward_f32(x, T, D, a[10], rms1_eps, a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7], a[8], a[9],
                          n_q, n_kv, head_dim, causal, rope_theta, a[11], rms2_eps, router_w, router_b,
                          ptrs, NULL, ptrs + E, NULL, ptrs + 2 * E, NULL, E, top_k, F, scratch_attn,
                          scratch_moe, reuse_idx, reuse_p);
  free(ptrs); free(scratch_attn); free(scratch_moe);
  ref_prof_clear();
  return 0;
}
