/*
 * moe_mkbin.c — writes a random-init Qwen3-MoE-shaped model as a .bin
 * weight file, in the layout that export.py --outdir followed by
 * merge_dir.py produces (export.py:130-178, merge_dir.py:34-43): the header
 * count is the number of original tensors, and each quantised expert
 * projection is two records, .scale then .q8/.q4.
 *
 *   moe_mkbin --out FILE [--layers 48] [--quant q8|q4|none] [--seed 1]
 *             [--std 0.02] [--d-model 2048] [--n-q 32] [--n-kv 4]
 *             [--head-dim 128] [--d-ff 768] [--experts 128] [--vocab 151936]
 *             [--tied] [--count tensors|records]
 *
 * --count records writes the number of records as the header count instead:
 * merge_bins.py (merge_bins.py:14-37) reads exactly that many records from
 * each input, so only files counted this way pass through it whole.
 * Tensor order follows the model's state dict: embed_tokens; per layer
 * q/k/v/o_proj, q_norm, k_norm, mlp.gate, experts e = 0..E-1 gate/up/down,
 * input_layernorm, post_attention_layernorm; model.norm; lm_head (absent
 * with --tied). Every tensor is N(0, std) from the counter-based stream of
 * moe_synth_normal_host with the tensor ids of mh_synth (include/moe_host.h),
 * and the experts are quantised by moe_quantize_rowwise_*_host. A file
 * written here and loaded by mh_load_bin therefore holds the weights that
 * mh_synth draws on the GPU, except where the device's double-precision
 * log/cos and glibc's differ enough to change a value's float rounding
 * (expected a few values in 10^9).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/moe_cuda.h"

static uint64_t stream_seed(uint64_t seed, uint64_t layer, uint64_t tid) {
  return seed * 1000003ull + layer * 1009ull + tid;
}

typedef struct {
  MoeBinWriter* w;
  uint64_t seed;
  float std;
  float* buf;
  void* qbuf;
  float* sbuf;
  int quant;      /* 0 none, 2 q8, 3 q4 */
} Ctx;

static int put_f32(Ctx* c, const char* name, uint64_t layer, uint64_t tid, int ndim, const int* shape) {
  size_t n = 1;
  for (int d = 0; d < ndim; ++d) n *= (size_t)shape[d];
  moe_synth_normal_host(stream_seed(c->seed, layer, tid), 0, n, c->std, c->buf);
  return moe_bin_put(c->w, name, 0, ndim, shape, c->buf);
}

static int put_expert(Ctx* c, const char* name, uint64_t layer, uint64_t tid, int rows, int cols) {
  const int shape[2] = {rows, cols};
  if (c->quant == 0) return put_f32(c, name, layer, tid, 2, shape);
  moe_synth_normal_host(stream_seed(c->seed, layer, tid), 0, (size_t)rows * cols, c->std, c->buf);
  int rc = c->quant == MOE_DTYPE_Q8
               ? moe_quantize_rowwise_q8_host(c->buf, rows, cols, (int8_t*)c->qbuf, c->sbuf)
               : moe_quantize_rowwise_q4_host(c->buf, rows, cols, (uint8_t*)c->qbuf, c->sbuf);
  if (rc) return rc;
  char k[300];
  snprintf(k, sizeof(k), "%s.scale", name);
  if ((rc = moe_bin_put(c->w, k, 0, 1, &rows, c->sbuf))) return rc;
  snprintf(k, sizeof(k), "%s.%s", name, c->quant == MOE_DTYPE_Q8 ? "q8" : "q4");
  const int qshape[2] = {rows, c->quant == MOE_DTYPE_Q8 ? cols : cols / 2};
  return moe_bin_put(c->w, k, c->quant == MOE_DTYPE_Q8 ? 2 : 3, 2, qshape, c->qbuf);
}

int main(int argc, char** argv) {
  const char* out = NULL;
  int layers = 48, D = 2048, nq = 32, nkv = 4, hd = 128, F = 768, E = 128, V = 151936, tied = 0, by_records = 0;
  Ctx c = {0};
  c.seed = 1; c.std = 0.02f; c.quant = MOE_DTYPE_Q8;
  for (int i = 1; i < argc; ++i) {
    const char* a = argv[i];
    if (!strcmp(a, "--tied")) { tied = 1; continue; }
    const char* v = i + 1 < argc ? argv[++i] : NULL;
    if (!v) { fprintf(stderr, "missing value after %s\n", a); return 2; }
    if (!strcmp(a, "--out")) out = v;
    else if (!strcmp(a, "--layers")) layers = atoi(v);
    else if (!strcmp(a, "--quant")) c.quant = !strcmp(v, "q4") ? MOE_DTYPE_Q4 : !strcmp(v, "none") ? 0 : MOE_DTYPE_Q8;
    else if (!strcmp(a, "--seed")) c.seed = strtoull(v, NULL, 10);
    else if (!strcmp(a, "--std")) c.std = (float)atof(v);
    else if (!strcmp(a, "--d-model")) D = atoi(v);
    else if (!strcmp(a, "--n-q")) nq = atoi(v);
    else if (!strcmp(a, "--n-kv")) nkv = atoi(v);
    else if (!strcmp(a, "--head-dim")) hd = atoi(v);
    else if (!strcmp(a, "--d-ff")) F = atoi(v);
    else if (!strcmp(a, "--experts")) E = atoi(v);
    else if (!strcmp(a, "--vocab")) V = atoi(v);
    else if (!strcmp(a, "--count")) by_records = !strcmp(v, "records");
    else { fprintf(stderr, "unknown option %s\n", a); return 2; }
  }
  if (!out || layers < 1 || D < 2 || nq < 1 || nkv < 1 || hd < 2 || F < 2 || E < 1 || V < 1) {
    fprintf(stderr, "usage: moe_mkbin --out FILE [--layers N] [--quant q8|q4|none] ...\n");
    return 2;
  }
  size_t big = (size_t)V * D;
  if ((size_t)nq * hd * D > big) big = (size_t)nq * hd * D;
  if ((size_t)F * D > big) big = (size_t)F * D;
  c.buf = (float*)malloc(sizeof(float) * big);
  c.qbuf = malloc((size_t)F * D);   /* the largest expert projection, as int8 */
  c.sbuf = (float*)malloc(sizeof(float) * (size_t)(F > D ? F : D));
  if (!c.buf || !c.qbuf || !c.sbuf) { fprintf(stderr, "out of host memory\n"); return 1; }
  const uint32_t per_expert = c.quant ? 2 : 1;   /* records per expert projection */
  const uint32_t count = 1 + (uint32_t)layers * (9 + 3 * (uint32_t)E * (by_records ? per_expert : 1)) + 1 +
                         (tied ? 0 : 1);
  c.w = moe_bin_create(out, count);
  if (!c.w) { fprintf(stderr, "%s\n", moe_cuda_last_error()); return 1; }
  int rc = 0;
  char k[256];
  const int emb_shape[2] = {V, D}, dvec[1] = {D}, hvec[1] = {hd};
  rc = put_f32(&c, "model.embed_tokens.weight", 65535, 0, 2, emb_shape);
  for (int L = 0; L < layers && !rc; ++L) {
    const int sq[2] = {nq * hd, D}, skv[2] = {nkv * hd, D}, so[2] = {D, nq * hd}, sr[2] = {E, D};
    static const char* const attn[4] = {"q_proj", "k_proj", "v_proj", "o_proj"};
    const int* ashape[4] = {sq, skv, skv, so};
    for (int j = 0; j < 4 && !rc; ++j) {
      snprintf(k, sizeof(k), "model.layers.%d.self_attn.%s.weight", L, attn[j]);
      rc = put_f32(&c, k, L, 100000 + j, 2, ashape[j]);
    }
    snprintf(k, sizeof(k), "model.layers.%d.self_attn.q_norm.weight", L);
    if (!rc) rc = put_f32(&c, k, L, 100004, 1, hvec);
    snprintf(k, sizeof(k), "model.layers.%d.self_attn.k_norm.weight", L);
    if (!rc) rc = put_f32(&c, k, L, 100005, 1, hvec);
    snprintf(k, sizeof(k), "model.layers.%d.mlp.gate.weight", L);
    if (!rc) rc = put_f32(&c, k, L, 0, 2, sr);
    static const char* const proj[3] = {"gate_proj", "up_proj", "down_proj"};
    for (int e = 0; e < E && !rc; ++e)
      for (int j = 0; j < 3 && !rc; ++j) {
        snprintf(k, sizeof(k), "model.layers.%d.mlp.experts.%d.%s.weight", L, e, proj[j]);
        rc = put_expert(&c, k, L, 2 + 3 * (uint64_t)e + j, j < 2 ? F : D, j < 2 ? D : F);
      }
    snprintf(k, sizeof(k), "model.layers.%d.input_layernorm.weight", L);
    if (!rc) rc = put_f32(&c, k, L, 100006, 1, dvec);
    snprintf(k, sizeof(k), "model.layers.%d.post_attention_layernorm.weight", L);
    if (!rc) rc = put_f32(&c, k, L, 100007, 1, dvec);
  }
  if (!rc) rc = put_f32(&c, "model.norm.weight", 65535, 1, 1, dvec);
  if (!rc && !tied) rc = put_f32(&c, "lm_head.weight", 65535, 2, 2, emb_shape);
  const int rc2 = moe_bin_finish(c.w);
  if (rc || rc2) { fprintf(stderr, "moe_mkbin: %s\n", moe_cuda_last_error()); return 1; }
  free(c.buf); free(c.qbuf); free(c.sbuf);
  return 0;
}
