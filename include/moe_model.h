/*
 * moe_model.h — the call surface of moe.cc's model.c, served by
 * libmoe_host.so: the same two functions with the same parameter lists and
 * structs, with attention, norms and the head on the CPU in fp32 (the
 * reference's arithmetic, bit for bit) and the MoE block on the GPU.
 *
 * Replaces:
 *   layer_forward_f32  model.c:38-58 (body :59-190)
 *   model_forward_f32  model.c:192-198 (body :199-252)
 * The reference file does not build as shipped (it lacks <stdio.h> for
 * model.h and the static helpers it calls live in test_model_trace.c); these
 * are its semantics as written:
 *   - every layer: rmsnorm(x) with rms1_eps; Q/K/V projections (+ biases);
 *     per-head Q/K RMSNorm with eps 1e-6 when both qn and kn are given; RoPE
 *     from position 0; scores over all T keys (causal: later keys -inf);
 *     softmax; context; output projection (+ bias); x += attn_out;
 *     x_norm2 = rmsnorm(x) with rms2_eps; router logits (+ bias); top-k by
 *     repeated arg-max (ties to the lower expert index, NaN never chosen);
 *     softmax over the chosen logits; per token and slot j in order,
 *     x += p_j * down(silu(gate x_norm2) * up x_norm2) added straight into x.
 *   - model_forward_f32: embeddings, the layers with eps 1e-6 and the
 *     config's causal / rope_theta / top_k, final rmsnorm (eps 1e-6), logits
 *     of every row [T][vocab] (lm_head, or tok_emb when lm_head is NULL),
 *     then softmax per row if apply_softmax.
 *
 * Experts are fp32 (Wg/Wu/Wd, as model.c requires; the biases bg/bu/bd are
 * ignored, as model.c ignores them). On the first call for a layer its
 * experts and router are copied to the GPU and kept there, keyed by the
 * router_w and Wg[0] pointers; moe_model_release() frees those copies (call
 * it before freeing or reusing the weight memory). The library initialises
 * CUDA device 0 itself if moe_cuda_init has not been called.
 *
 * Scratch: layer_forward_f32 uses scratch_attn for its first
 * T*(n_q*dh + 2*n_kv*dh) + T*T + T*n_q*dh + 2*T*D floats, the documented
 * size; scratch_moe is not needed (may be NULL). reuse_topk_idx /
 * reuse_topk_p, when both are non-NULL, are the routing to use ([T][topk]),
 * as in model.c:139-141.
 *
 * Errors: the reference has no error returns; a failure here prints the
 * library's message to stderr and aborts.
 */
#ifndef MOE_MODEL_H
#define MOE_MODEL_H

#include <stddef.h>
#include <stdint.h>

#include "moe_cuda.h"   /* QuantizedWeight */

#ifdef __cplusplus
extern "C" {
#endif

/* The structs of model.h:9-59, same layout. When the reference's model.h is
 * included first, its definitions are used. */
#ifndef MODEL_H
typedef struct {
  int d_model;
  int n_layers;
  int head_dim;
  int n_q;
  int n_kv;
  int d_ff;
  int n_experts;
  int top_k;
  int vocab_size;
  int causal;
  float rope_theta;
  float rms_eps;
} QwenConfig;

typedef struct {
  const float* Wq; const float* bq;
  const float* Wk; const float* bk;
  const float* Wv; const float* bv;
  const float* Wo; const float* bo;
  const float* q_norm;
  const float* k_norm;
  const float* rms1_w;
  const float* rms2_w;
  const float* router_w;
  const float* router_b;
  const float** Wg; const float** bg;
  const float** Wu; const float** bu;
  const float** Wd; const float** bd;
  QuantizedWeight* Wg_q;
  QuantizedWeight* Wu_q;
  QuantizedWeight* Wd_q;
  int experts_quantized;
} QwenLayerWeights;

typedef struct {
  const float* tok_emb;
  const float* final_norm_w;
  const float* lm_head;
  QwenLayerWeights* layers;
} QwenWeights;
#endif

/* model.c:38-58 */
void layer_forward_f32(
  float* x, int T, int D,
  const float* rms1_w, float rms1_eps,
  const float* Wq, const float* bq,
  const float* Wk, const float* bk,
  const float* Wv, const float* bv,
  const float* Wo, const float* bo,
  const float* qn, const float* kn,
  int n_q, int n_kv, int head_dim, int causal, float rope_theta,
  const float* rms2_w, float rms2_eps,
  const float* router_w, const float* router_b,
  const float** Wg, const float** bg,
  const float** Wu, const float** bu,
  const float** Wd, const float** bd,
  int n_experts, int topk, int d_ff,
  float* scratch_attn,
  float* scratch_moe,
  int*   reuse_topk_idx,
  float* reuse_topk_p);

/* model.c:192-198 */
void model_forward_f32(
  const int* ids, int T,
  const QwenConfig* cfg,
  const QwenWeights* w,
  int apply_softmax,
  float* out_logits);

/* Frees the GPU copies of the layers the two functions above uploaded. No
 * reference counterpart (the reference keeps no device state). */
void moe_model_release(void);

#ifdef __cplusplus
}
#endif
#endif /* MOE_MODEL_H */
