/*
 * moe_host.h — C host driver around libmoe_cuda: a KV-cached, batched
 * greedy decoder for Qwen3-MoE-shaped models, attention on the CPU in fp32
 * and the MoE block resident on the GPU (moe_ffn).
 *
 * Replaces the reference's full-model loop (test_model_trace.c:526-596
 * model_forward_f32 and the generation loop of main, :703-745), which
 * recomputes the whole prefix at every step. Here each step runs only the
 * new tokens and keeps K/V per layer. Attention is causal and every row of
 * the reference's computation depends only on earlier rows, so the cached
 * step computes the same logits bit for bit: the CPU arithmetic restates
 * the reference's matmul_f32, rmsnorm_forward_f32, per-head Q/K RMSNorm,
 * rope_apply_inplace_f32_gqa and attention softmax in their operation order
 * (:213-427), and moe_ffn reproduces :463-517.
 *
 * A model holds `batch` sequences that advance in lockstep (the same number
 * of new tokens per step); each step's MoE call covers all of them
 * (batch x new tokens rows), which is what batched decode buys on the GPU.
 *
 * Errors: status codes (MOE_OK / MOE_ERR_* of moe_cuda.h), message in
 * mh_last_error() (per calling thread). No function exits the process.
 */
#ifndef MOE_HOST_H
#define MOE_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* QwenConfig (model.h:9-22); causal is always 1 and top_k is 8. */
typedef struct {
  int d_model, n_layers, head_dim, n_q, n_kv, d_ff, n_experts, vocab_size;
  float rope_theta, rms_eps;
} MhConfig;

/* One layer's fp32 attention and norm weights (QwenLayerWeights,
 * model.h:34-46), host pointers borrowed by the model. Biases, q_norm and
 * k_norm may be NULL. Wq [n_q*hd][D], Wk/Wv [n_kv*hd][D], Wo [D][n_q*hd]. */
typedef struct {
  const float *Wq, *bq, *Wk, *bk, *Wv, *bv, *Wo, *bo;
  const float *q_norm, *k_norm, *rms1_w, *rms2_w;
} MhLayerWeights;

typedef struct MhModel MhModel;

/* A model for `batch` sequences of at most max_ctx positions: KV caches of
 * n_layers x batch x max_ctx x n_kv*head_dim floats for K and for V. Weights
 * are set by mh_set_* (borrowed), mh_load_bin or mh_synth (owned).
 * moe_layer_base: moe_cuda layer id of model layer 0 (layer l uses
 * moe_layer_base + l). Needs moe_cuda_init for anything that reaches the GPU. */
MhModel* mh_create(const MhConfig* cfg, int batch, int max_ctx, int moe_layer_base);
void mh_free(MhModel* m);
const char* mh_last_error(void);

int mh_set_globals(MhModel* m, const float* tok_emb, const float* final_norm_w,
                   const float* lm_head /* NULL: tied to tok_emb */);
int mh_set_layer(MhModel* m, int layer, const MhLayerWeights* w);

/* Config of a .bin weight file, inferred as load_all_weights does
 * (model.h:107-160): sizes from the tensor shapes, layers counted by probing
 * q_proj, experts by probing layer 0's down_proj, rope_theta 1e7, eps 1e-6.
 * Host only. */
int mh_config_from_bin(const char* path, MhConfig* cfg);
/* All weights of the file: attention/norm tensors into host memory owned by
 * the model (names of model.h:162-210), the MoE layers resident on the GPU
 * (moe_cuda_load_bin_layer_h). */
int mh_load_bin(MhModel* m, const char* path);
/* Random-init weights: every fp32 tensor ~ N(0, std) from the counter-based
 * stream of moe_synth_normal_* (drawn on the GPU, copied to the host), the
 * experts drawn on the GPU and quantised there (expert_dtype 2 = Q8, 3 = Q4),
 * router ~ N(0, std). Stream of tensor `tid` of layer l: seed*1000003 +
 * l*1009 + tid (tid 0 router, 2+3e/3+3e/4+3e expert e gate/up/down,
 * 100000+0..7 Wq, Wk, Wv, Wo, q_norm, k_norm, rms1, rms2); globals use layer
 * 65535 (tid 0 tok_emb, 1 final norm, 2 lm_head). */
int mh_synth(MhModel* m, uint64_t seed, int expert_dtype, float std);

/* Current position (tokens already in the caches) and a reset to 0. */
int mh_pos(const MhModel* m);
void mh_reset(MhModel* m);
/* Fill every cache position [0, ctx) with N(0, std) (stream `seed`) and set
 * the position to ctx: a prefilled context for decode measurements. */
int mh_fill_kv(MhModel* m, int ctx, uint64_t seed, float std);

/* Feed T new tokens per sequence (ids [batch][T]) and return the logits of
 * each sequence's last token (logits [batch][vocab], before softmax). */
int mh_step(MhModel* m, const int* ids, int T, float* logits);

/* Greedy decode: prompts [batch][prompt_len] from position 0, then `steps`
 * tokens per sequence, each the argmax of softmax(logits) with the first
 * maximum winning (test_model_trace.c:723-731); out [batch][steps]. */
int mh_generate(MhModel* m, const int* prompts, int prompt_len, int steps, int* out);

/* The greedy choice of mh_generate for each sequence's logits row
 * (logits [batch][vocab], softmaxed in place); ids [batch]. */
int mh_pick_greedy(const MhModel* m, float* logits, int* ids);

/* The pieces of one step, for callers that drive the layers themselves.
 * mh_embed: x [batch*T][D] from ids. mh_attention: x -> x_after =
 * x + attn(rmsnorm1(x)) and x_norm2 = rmsnorm2(x_after) for layer l over the
 * T new tokens at the current position, appending their K/V to the cache.
 * mh_moe: x_after -> x_after + moe(x_norm2) on the GPU. mh_head: logits
 * of rows (t = T-1) of each sequence. mh_advance: position += T. */
int mh_embed(MhModel* m, const int* ids, int T, float* x);
int mh_attention(MhModel* m, int layer, const float* x, int T, float* x_after, float* x_norm2);
int mh_moe(MhModel* m, int layer, const float* x_norm2, float* x_after, int T);
int mh_head(MhModel* m, const float* x, int T, float* logits);
int mh_advance(MhModel* m, int T);

/* Expert parallelism: this process is rank ep_rank of the ep_world group it
 * passed to moe_cuda_init; the model's MoE layers hold only this rank's
 * experts (every upload path shards them), and the model's `batch`
 * sequences are this rank's own. mh_ep_setup allocates the exchange for up
 * to max_rows_per_call rows per MoE call (batch x new tokens; larger steps
 * run in chunks of that size) and writes this rank's 64-byte handle; the
 * caller exchanges the handles (rank order) and passes all of them to
 * mh_ep_connect. From then on every MoE block runs moe_ffn_ep: all ranks
 * must step together, with the same batch and token counts (the reference
 * runs on one CPU and has no counterpart). */
int mh_ep_setup(MhModel* m, int max_rows_per_call, void* handle_out);
int mh_ep_connect(MhModel* m, const void* handles);

/* Accumulated wall time of the MoE calls per layer since the last reset
 * (ms[n_layers], calls[n_layers]; either may be NULL) and of the CPU part. */
int mh_timing(const MhModel* m, double* moe_ms, long* moe_calls, double* cpu_ms);
void mh_timing_reset(MhModel* m);

#ifdef __cplusplus
}
#endif
#endif /* MOE_HOST_H */
