/*
 * moe_cuda.h — C-ABI of libmoe_cuda.so, the B200 (sm_100a) implementation of
 * moe.cc's MoE expert-FFN hot path.
 *
 * Plain C99: pointers, sizes and int status codes only. A C host that today
 * links kernels.o (moe.cc Makefile:8-9) links libmoe_cuda.so instead and keeps
 * calling matmul_adaptive() unchanged; the fused moe_ffn() replaces the whole
 * MoE block of layer_forward_f32 (test_model_trace.c:463-517).
 *
 * Arithmetic contract (identical to the reference, not "dequant(W)·x"):
 *   Q8:  C[m,n] = ((float)Σ_k (int32)(A[m,k]*127f) * q[n,k] / 127f) * s[n]
 *   Q4:  C[m,n] = ((float)Σ_k (int32)(A[m,k]*7f) * (nib[n,k]-8) / 7f) * s[n]
 * with truncation toward zero, exact int32 accumulation (two's-complement
 * wrap), IEEE round-to-nearest divide and multiply (kernels.c:51-74, 96-128).
 *
 * Status codes: every int-returning entry point returns MOE_OK (0) or one of
 * the MOE_ERR_* codes below; moe_cuda_last_error() gives a message. The
 * void-returning reference-shaped entry points (matmul_f32_q8/_q4,
 * matmul_adaptive) cannot return a status: on failure they print the message
 * to stderr and abort(), because the reference host has no error path and a
 * silently wrong result is worse than a crash.
 *
 * Threading: one host thread per device; all device work is ordered on the
 * stream passed in (NULL = the legacy default stream).
 */
#ifndef MOE_CUDA_H
#define MOE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same layout as moe.cc model.h:26-32, so a QwenLayerWeights' Wg_q/Wu_q/Wd_q
 * arrays can be passed as they are. */
#ifndef QUANTIZED_WEIGHT_DEFINED
typedef struct {
  const int8_t* q;      /* Q8: int8 [rows][cols]; Q4: uint8 [rows][cols/2] */
  const float* s;       /* per-row fp32 scale [rows] */
  int rows, cols;       /* logical shape (Q4: cols = 2 * packed bytes) */
  int dtype;            /* 2 = Q8, 3 = Q4 (TensorBin dtype enum) */
} QuantizedWeight;
#define QUANTIZED_WEIGHT_DEFINED
#endif

#define MOE_OK               0
#define MOE_ERR_INVALID      1  /* bad argument / shape / dtype */
#define MOE_ERR_CUDA         2  /* a CUDA runtime call failed */
#define MOE_ERR_NOT_INIT     3  /* moe_cuda_init() not called / layer missing */
#define MOE_ERR_RANGE        4  /* reserved: no entry point returns it (an
                                   activation outside the fast kernels' integer
                                   range is recomputed exactly on the device) */
#define MOE_ERR_UNSUPPORTED  5  /* valid for the reference, not built here */
#define MOE_ERR_NOMEM        6  /* device allocation failed */

#define MOE_DTYPE_F32 0   /* unquantised fp32 experts (moe_cuda_upload_layer_f32) */
#define MOE_DTYPE_Q8 2
#define MOE_DTYPE_Q4 3

/* moe_ffn flags */
#define MOE_FFN_HOST_PTRS   0x1 /* x/out/topk pointers are host memory: the
                                   call copies in, computes, copies out and
                                   synchronises the stream */
#define MOE_FFN_DEVICE_PTRS 0x0 /* all pointers are device memory; async */
#define MOE_FFN_FORCE_GEMV  0x4 /* always use the decode (GEMV) kernels */
#define MOE_FFN_FORCE_GEMM  0x8 /* always use the grouped tcgen05 GEMM */
#define MOE_FFN_SEQ_RESIDUAL 0x10 /* add p*y into x_inout one slot at a time,
                                     x = ((x + p0 y0) + p1 y1) + ..., as
                                     model.c:188 does, instead of
                                     x + (p0 y0 + p1 y1 + ...) as
                                     test_model_trace.c:513,517 */
#define MOE_FFN_GIVEN_TOPK  0x20 /* topk_idx_out / topk_p_out are inputs: the
                                    routing to use (model.c:139-141 reuse_topk),
                                    no router or top-k is computed */

/* ---- runtime -------------------------------------------------------------
 * No reference counterpart (moe.cc has no device); the reference's process
 * state is only io.c's progress globals (io.c:14-33).
 * ep_world/ep_rank: expert-parallel group. Rank r owns experts
 * [r*E/ep_world, (r+1)*E/ep_world) of every layer it uploads. nccl_uid is
 * reserved and must be NULL (the cross-rank exchange is driven by the caller
 * through moe_ffn_partial + its own communicator). */
int moe_cuda_init(int device, int ep_world, int ep_rank, const void* nccl_uid);
int moe_cuda_shutdown(void);
const char* moe_cuda_last_error(void);
/* Synchronise the device and report (then clear) any error a kernel flagged
 * asynchronously: MOE_ERR_CUDA when a bounded device-side wait ran out (a copy
 * that never landed, or another rank's flag that was not raised in time). */
int moe_cuda_check_status(void);

/* ---- reference kernel surface (kernels.c / kernels.h) --------------------
 * Host pointers, synchronous. If B_q/B_s are host pointers previously given
 * to moe_cuda_upload_layer (or moe_cuda_upload_layer_dev), the resident device
 * copy is used; otherwise the weight is copied for this call only. */
/* replaces static matmul_f32_q8, kernels.c:51 (same parameter list) */
void matmul_f32_q8(const float* A, const int8_t* B_q, const float* B_s,
                   float* C, int M, int N, int K);
/* replaces static matmul_f32_q4, kernels.c:96 (same parameter list). K must
 * be even: with odd K the reference reads the last weight byte's low nibble
 * and then one byte past the packed row (kernels.c:108,116-119), memory it
 * does not own; this library returns MOE_ERR_UNSUPPORTED for odd K instead
 * (the host-pointer form aborts with that message). */
void matmul_f32_q4(const float* A, const uint8_t* B_q, const float* B_s,
                   float* C, int M, int N, int K);
/* replaces matmul_adaptive, kernels.h:16-17 / kernels.c:149-181:
 * W_q_ptr == NULL -> sequential fp32 dot; dtype 2/3 -> Q8/Q4; any other
 * dtype -> C zero-filled (kernels.c:172-180). */
void matmul_adaptive(const float* A, const float* W_fp32, const void* W_q_ptr,
                     float* C, int M, int N, int K);

/* Device-pointer, stream-ordered forms of the three above (same math).
 * stream is a cudaStream_t (NULL = default stream). */
int moe_matmul_q8_dev(const float* A, const int8_t* B_q, const float* B_s,
                      float* C, int M, int N, int K, void* stream);
int moe_matmul_q4_dev(const float* A, const uint8_t* B_q, const float* B_s,
                      float* C, int M, int N, int K, void* stream);
int moe_matmul_f32_dev(const float* A, const float* W, float* C,
                       int M, int N, int K, void* stream);
/* Many independent GEMVs of one activation row against n_mat Q8/Q4 matrices
 * of identical shape (the "all experts' gate matrices in one launch" form of
 * config C1): C[i][n] = matmul(A[1,K], W_i[N,K]). W_q/W_s are device arrays
 * of n_mat device pointers. No reference counterpart (one loop of calls to
 * matmul_adaptive with M=1 in the reference). */
int moe_matmul_batched_dev(const float* A, const void* const* W_q,
                           const float* const* W_s, float* C, int n_mat,
                           int N, int K, int dtype, void* stream);

/* Allocation-free form of moe_matmul_q8_dev / moe_matmul_q4_dev (dtype 2 or 3),
 * for callers that must not allocate GPU memory at call time (code inside a
 * memory-pool or allocator callback, hosts whose device memory is entirely
 * reserved up front, latency-critical paths that cannot take cudaMalloc's
 * implicit synchronisation). No counterpart in the reference. Same results as
 * moe_matmul_q8_dev/_q4_dev, bit for bit, for any input magnitude (K = 0
 * gives zeros). Scratch is a fixed 1 MiB + 16.25 KiB device array inside the
 * library (held by every GPU that loads it until exit): shapes on the fast
 * path (packed rows a multiple of 16 bytes, B_q 16-byte aligned) need
 * M <= 4096 and M*K <= 524288, and larger ones return MOE_ERR_INVALID; other
 * shapes use no scratch. Needs no moe_cuda_init. The first call on each
 * device is its set-up: it resolves the array's address and, with CUDA's lazy
 * module loading, loads the library's kernels, which allocates device memory;
 * make that first call before any stream capture and outside any region that
 * must not allocate. Not valid across a cudaDeviceReset. All calls share the
 * array: calls whose GPU work overlaps race on it. */
int moe_matmul_q_dev_noalloc(const float* A, const void* B_q, const float* B_s,
                             float* C, int M, int N, int K, int dtype,
                             void* stream);

/* ---- quantisers (export.py:23-36) -----------------------------------------
 * Bit-exact with export._rowwise_q8 / _rowwise_q4: s = max(max|row|,1e-8)/127
 * (or /7), q = round-half-even(w/s) (Q4: clamped to [-8,7], +8, two nibbles a
 * byte, even column in the low nibble). Device pointers. */
int moe_quantize_rowwise_q8_dev(const float* W, int rows, int cols,
                                int8_t* q, float* s, void* stream);
int moe_quantize_rowwise_q4_dev(const float* W, int rows, int cols,
                                uint8_t* q, float* s, void* stream);

/* ---- weight residency (model.h:220-305 + io.c:193-320) --------------------
 * Copies one layer's experts (host QuantizedWeight arrays of length E, as in
 * QwenLayerWeights.Wg_q/Wu_q/Wd_q, model.h:55-57) and router (model.h:44-45;
 * router_b may be NULL, model.h:217-218) into device memory: one slab per
 * expert holding [gate q | up q | down q | gate s | up s | down s], every
 * part 128-byte aligned. Under expert parallelism only this rank's experts
 * are copied. The host q/s pointers are remembered, so later matmul_f32_q8/
 * _q4/matmul_adaptive calls on them run on the resident copy. */
int moe_cuda_upload_layer(int layer, const QuantizedWeight* Wg,
                          const QuantizedWeight* Wu, const QuantizedWeight* Wd,
                          const float* router_w, const float* router_b, int E);
/* Same, but every q/s pointer in Wg/Wu/Wd and router_w/router_b is DEVICE
 * memory (e.g. the output of moe_quantize_rowwise_*_dev). Sizes as above. */
int moe_cuda_upload_layer_dev(int layer, const QuantizedWeight* Wg,
                              const QuantizedWeight* Wu,
                              const QuantizedWeight* Wd,
                              const float* router_w, const float* router_b,
                              int E);
/* A layer with unquantised fp32 experts, as model.c's layer_forward_f32 takes
 * them (QwenLayerWeights Wg/Wu/Wd, model.h:41-43, used at model.c:172-187):
 * Wg[e], Wu[e] host [F][D], Wd[e] host [D][F], e < E; router_w [E][D],
 * router_b [E] or NULL; top_k experts per token (1..32, <= E). moe_ffn then
 * runs the fp32 expert FFN (each output one sequential fp32 chain in k order,
 * as matmul_f32, test_model_trace.c:213-227). No expert parallelism. */
int moe_cuda_upload_layer_f32(int layer, const float* const* Wg, const float* const* Wu,
                              const float* const* Wd, const float* router_w,
                              const float* router_b, int E, int D, int F, int top_k);
int moe_cuda_free_layer(int layer);
/* Bytes of device memory the layer's expert slabs occupy on this rank. */
size_t moe_cuda_layer_bytes(int layer);

/* ---- weight files -------------------------------------------------------------
 * The reference's .bin weight file (export.py _save_tensor, :8-21; read by
 * io.c:193-285 and model.h:212-305): magic "QW3W\0\1", a u32 count, then
 * records (u32 name length, name, u32 dtype, u32 ndim, u32 shape[ndim], data).
 *
 * moe_bin_layer_info: the MoE shape of layer src_layer of the file (E experts,
 * hidden D, expert width F, dtype 2 = Q8 / 3 = Q4, has_bias 1 when an f32
 * model.layers.L.mlp.gate.bias is present). Host only: needs no GPU and no
 * moe_cuda_init. Any output pointer may be NULL.
 *
 * moe_cuda_load_bin_layer: reads layer src_layer's router (and bias) and this
 * rank's experts from the file and makes them resident as `layer`, as
 * moe_cuda_upload_layer does (replaces load_model_weights' per-layer MoE part,
 * model.h:212-305, for a caller that hands the layer to moe_ffn). Only the
 * record headers of the rest of the file are read. No host pointers are
 * registered for the matmul_* drop-ins.
 *
 * Both return MOE_ERR_INVALID for a malformed or truncated file, a missing
 * tensor or a shape/dtype mismatch (the reference exits the process),
 * MOE_ERR_UNSUPPORTED for unquantised (f32) experts. */
int moe_bin_layer_info(const char* path, int src_layer, int* E, int* D, int* F,
                       int* dtype, int* has_bias);
int moe_cuda_load_bin_layer(const char* path, int src_layer, int layer);

/* The same over an open file, indexed once (bin_load / bin_find, io.h:20-22,
 * without reading the data). moe_bin_open returns NULL on error (message in
 * moe_cuda_last_error). moe_bin_find gives a record's dtype (0 f32, 1 f16,
 * 2 i8, 3 packed i4), ndim, shape (up to 8 entries) and data bytes;
 * moe_bin_read copies its data into dst (nbytes must equal the record's).
 * A repeated name resolves to its first record. A handle may be shared by
 * threads (reads are serialised). */
typedef struct MoeBin MoeBin;
MoeBin* moe_bin_open(const char* path);
void moe_bin_close(MoeBin* bin);
int moe_bin_find(MoeBin* bin, const char* name, int* dtype, int* ndim, int* shape,
                 size_t* nbytes);
int moe_bin_read(MoeBin* bin, const char* name, void* dst, size_t nbytes);
int moe_bin_layer_info_h(MoeBin* bin, int src_layer, int* E, int* D, int* F,
                         int* dtype, int* has_bias);
int moe_cuda_load_bin_layer_h(MoeBin* bin, int src_layer, int layer);

/* Writing the format: moe_bin_create writes the magic and `count`, then
 * moe_bin_put appends one record per call (dtype 0 f32, 1 f16, 2 i8, 3
 * packed i4; data of prod(shape) x 4/2/1/1 bytes) and moe_bin_finish closes
 * the file. export.py and merge_dir.py (:34-43) write the number of original
 * tensors as the count, while a quantised tensor contributes two records,
 * .scale then .q8/.q4 (export.py:197-206); readers go to end of file. */
typedef struct MoeBinWriter MoeBinWriter;
MoeBinWriter* moe_bin_create(const char* path, uint32_t count);
int moe_bin_put(MoeBinWriter* w, const char* name, int dtype, int ndim,
                const int* shape, const void* data);
int moe_bin_finish(MoeBinWriter* w);

/* The quantisers above on host memory (same results bit for bit). */
int moe_quantize_rowwise_q8_host(const float* W, int rows, int cols, int8_t* q, float* s);
int moe_quantize_rowwise_q4_host(const float* W, int rows, int cols, uint8_t* q, float* s);

/* ---- fused MoE block --------------------------------------------------------
 * Replaces test_model_trace.c:463-517 (router matmul + bias, topk_desc,
 * top-k softmax, per-(token,k) gate/up/SiLU·up/down, k-ordered weighted
 * combine, residual add):
 *   x_inout[t] = x_inout[t] + Σ_{k=0..top_k-1} p[t,k] · down_e(silu(gate_e x)·up_e x)
 * x_norm2: [T][D] fp32 input to the experts; x_inout: [T][D] fp32, holds
 * x_after on entry and x on return (test_model_trace.c:517).
 * topk_idx_out/topk_p_out: optional [T][top_k] (NULL to skip), or with
 * MOE_FFN_GIVEN_TOPK the routing to use (inputs).
 * Any activation magnitude: the fast kernels carry trunc(127x) in 16 bits
 * (Q8, |x| < 258) and trunc(7x) in 8 bits (Q4); a token whose x, or the h of
 * one of its slots, leaves that range (or is NaN/inf) is marked, and an exact
 * int32 fix-up pass on the device recomputes its slots before the combine,
 * so every call returns the reference's result (the reference truncates with
 * no range limit, kernels.c:66, :113).
 * A slot with no expert (fewer than top_k logits that are neither NaN nor
 * -inf; the reference then reads an expert out of bounds) adds p * 0.
 * MOE_FFN_HOST_PTRS on page-locked host buffers (cudaHostAlloc,
 * cudaMallocHost, cudaHostRegister): x_norm2 is copied in, and the combine
 * kernel updates x_inout in place through its mapped address and writes the
 * top-k outputs to host memory, so no copies come back; pageable buffers are
 * copied both ways. Both give the same results.
 * With ep_world > 1 use moe_ffn_partial or moe_ffn_ep instead. */
int moe_ffn(int layer, const float* x_norm2, float* x_inout, int T,
            int* topk_idx_out, float* topk_p_out, int flags, void* stream);

/* Expert-parallel form: computes router/top-k on every rank (identical
 * results), and for this rank's experts only, writes y_slots[T*top_k][D]
 * (y of slot t*top_k+k, zero where the slot's expert lives on another rank)
 * and topk_p [T*top_k]. After the caller sums y_slots over ranks (a
 * reduce — exact, because exactly one rank contributes each slot), call
 * moe_ffn_combine to apply the k-ordered combine and residual. Device
 * pointers, async. */
int moe_ffn_partial(int layer, const float* x_norm2, int T, float* y_slots,
                    int* topk_idx_out, float* topk_p_out, void* stream);
int moe_ffn_combine(const float* y_slots, const float* topk_p, float* x_inout,
                    int T, int D, int top_k, void* stream);

/* ---- expert parallelism with both exchanges fused into the kernels --------
 * The multi-GPU form of the MoE block (the reference runs it on one CPU,
 * test_model_trace.c:463-517; no counterpart there). Rank r owns experts
 * [r*E/W, (r+1)*E/W) (moe_cuda_init's ep_world/ep_rank) and T_local tokens.
 * Per call, with no collective library involved:
 *   routing kernel  routes this rank's tokens, stores their truncated
 *                   activations and top-k into every rank's exchange buffer
 *                   (peer stores over NVLink), raises this rank's dispatch
 *                   flag at every rank, waits (bounded) for all ranks' flags
 *                   and builds the routing lists of its own experts over all
 *                   ranks' tokens;
 *   expert GEMMs    as in moe_ffn; the down projection's epilogue stores each
 *                   slot row into the exchange buffer of the rank owning the
 *                   slot's token, and its last CTA raises the combine flag
 *                   (when no token was marked out of range);
 *   exact fix-up    when some rank marked a token (x or h outside the fast
 *                   integer range), the experts' owners recompute its slots
 *                   exactly from the home rank's published inputs, store the
 *                   rows, then raise the combine flags;
 *   combine         waits (bounded) for all ranks' combine flags, then the
 *                   k-ordered combine + residual of this rank's tokens.
 * Each wait on another rank gives up after MOE_EP_WAIT_MS milliseconds
 * (environment, default 200; ranks must enter each call within that time of
 * one another) and reports MOE_ERR_CUDA through moe_cuda_check_status
 * instead of hanging; a fresh moe_cuda_ep_setup / moe_cuda_ep_connect on
 * every rank then starts over. Needs one GPU per rank. An entry of
 * ep_connect's table that holds this rank's own handle maps its own buffer
 * (a loopback group in one process, whose waits on that entry can only run
 * out; used to test the waits on one GPU).
 *   moe_cuda_ep_setup: allocate this rank's exchange buffers for up to
 *     max_tokens_local tokens per rank of width D with top_k slots each and
 *     write its 64-byte CUDA IPC handle to ipc_handle_out. Every rank calls
 *     it, then the ranks exchange the handles (e.g. an all-gather).
 *   moe_cuda_ep_connect: ipc_handles = ep_world handles of 64 bytes in rank
 *     order; maps the peers' buffers.
 *   moe_ffn_ep: x_norm2 = this rank's normalised tokens [T_local][D];
 *     x_inout = its residual stream [T_local][D], updated in place. Every
 *     rank calls it with the same layer and T_local. Tensor-core path only
 *     (Q8/Q4 layers, D and F multiples of 128) and at most 2048 routed slots
 *     (T_local * ep_world * top_k) per call, else MOE_ERR_UNSUPPORTED.
 *     Device pointers, async on `stream`. */
int moe_cuda_ep_setup(int max_tokens_local, int D, int top_k, void* ipc_handle_out);
int moe_cuda_ep_connect(const void* ipc_handles);
int moe_ffn_ep(int layer, const float* x_norm2, int T_local, float* x_inout,
               void* stream);

/* ---- profiling -------------------------------------------------------------
 * Per-kernel device time of moe_ffn / moe_ffn_partial (CUDA events recorded
 * on the launching stream around each launch). Counterpart of the
 * reference's PROF_START/PROF_ENDF profiler (test_model_trace.c:64-199).
 * moe_cuda_profile(1) clears and starts, (0) stops. moe_cuda_profile_read
 * synchronises and fills up to max_kernels entries: names (name_len bytes
 * each), total milliseconds and launch counts; returns the entry count. */
int moe_cuda_profile(int enable);
int moe_cuda_profile_read(int max_kernels, char* names, int name_len,
                          double* total_ms, long* launches);

/* ---- synthetic inputs -----------------------------------------------------
 * out[i] = std * N(0,1) sample i of the counter-based stream `seed`
 * (splitmix64 -> Box-Muller in double -> float), i = offset .. offset+n-1.
 * Host and device forms produce the same stream. Harness convenience only;
 * no reference counterpart. */
void moe_synth_normal_host(uint64_t seed, uint64_t offset, size_t n, float std,
                           float* out);
int moe_synth_normal_dev(uint64_t seed, uint64_t offset, size_t n, float std,
                         float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MOE_CUDA_H */
