/*
 * moe_generate.c — greedy decode over the C host driver (include/moe_host.h):
 * the full-model workloads of the MoE path, with the MoE block on the GPU
 * and attention on the host, timed per layer.
 *
 *   moe_generate [--bin FILE] [--layers 48] [--dtype q8|q4] [--batch 1]
 *                [--prompt 64] [--steps 256] [--ctx 4096] [--kv-fill 0]
 *                [--seed 1] [--device 0] [--ep-dir DIR] [--out FILE]
 *
 * Without --bin the model is the Qwen3-30B-A3B shape with random-init
 * weights (mh_synth: fp32 ~ N(0, 0.02), experts quantised on the GPU,
 * RoPE theta 1e6, eps 1e-6). The prompt is `prompt` uniform-random token ids
 * per sequence. --kv-fill N first fills positions [0, N) of every cache with
 * N(0, 1) and starts decoding after them (batched decode at a long context).
 * Prints one JSON line: decode tokens/s over all sequences, the prefill time,
 * and the MoE wall time per layer call (host-pointer moe_ffn, copies
 * included) against the host attention time.
 *
 * Expert parallelism: started as WORLD_SIZE processes (RANK, LOCAL_RANK in
 * the environment, e.g. by torchrun) with --ep-dir naming a directory all of
 * them can write, rank r runs on GPU LOCAL_RANK, holds experts
 * [r*E/W, (r+1)*E/W) of every layer and decodes batch/W of the sequences; the
 * MoE blocks run moe_ffn_ep. The ranks exchange their exchange-buffer handles
 * and meet at barriers through files in that directory. Rank 0 prints the
 * line, with decode tokens/s over all ranks' sequences.
 */
#include <errno.h>
#include <unistd.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "../../include/moe_cuda.h"
#include "../../include/moe_host.h"

static double now_ms(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

/* ---- file-based rendezvous of the expert-parallel ranks ---- */
static int wait_files(const char* dir, const char* tag, int world) {
  char path[4096];
  const double t0 = now_ms();
  for (int r = 0; r < world; ++r) {
    snprintf(path, sizeof(path), "%s/%s.%d", dir, tag, r);
    while (access(path, R_OK) != 0) {
      if (now_ms() - t0 > 600e3) { fprintf(stderr, "rendezvous: %s did not appear\n", path); return 1; }
      usleep(1000);
    }
  }
  return 0;
}

static int put_file(const char* dir, const char* tag, int rank, const void* data, size_t n) {
  char tmp[4096], path[4096];
  snprintf(tmp, sizeof(tmp), "%s/.%s.%d.tmp", dir, tag, rank);
  snprintf(path, sizeof(path), "%s/%s.%d", dir, tag, rank);
  FILE* f = fopen(tmp, "wb");
  if (!f || (n && fwrite(data, 1, n, f) != n)) { fprintf(stderr, "rendezvous: write %s: %s\n", tmp, strerror(errno)); return 1; }
  fclose(f);
  return rename(tmp, path) != 0;
}

static int barrier(const char* dir, const char* tag, int rank, int world) {
  return put_file(dir, tag, rank, NULL, 0) || wait_files(dir, tag, world);
}

static uint64_t splitmix(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

int main(int argc, char** argv) {
  const char* bin = NULL;
  const char* ep_dir = NULL;
  const char* out_path = NULL;    /* --out FILE: this rank's tokens to FILE.<rank> */
  int layers = 48, dtype = MOE_DTYPE_Q8, batch = 1, prompt = 64, steps = 256, ctx = 4096, kv_fill = 0, device = 0;
  unsigned long long seed = 1;
  for (int i = 1; i < argc; ++i) {
    const char* a = argv[i];
    const char* v = i + 1 < argc ? argv[i + 1] : NULL;
    if (!v) { fprintf(stderr, "missing value after %s\n", a); return 2; }
    if (!strcmp(a, "--bin")) bin = v;
    else if (!strcmp(a, "--layers")) layers = atoi(v);
    else if (!strcmp(a, "--dtype")) dtype = !strcmp(v, "q4") ? MOE_DTYPE_Q4 : MOE_DTYPE_Q8;
    else if (!strcmp(a, "--batch")) batch = atoi(v);
    else if (!strcmp(a, "--prompt")) prompt = atoi(v);
    else if (!strcmp(a, "--steps")) steps = atoi(v);
    else if (!strcmp(a, "--ctx")) ctx = atoi(v);
    else if (!strcmp(a, "--kv-fill")) kv_fill = atoi(v);
    else if (!strcmp(a, "--seed")) seed = strtoull(v, NULL, 10);
    else if (!strcmp(a, "--device")) device = atoi(v);
    else if (!strcmp(a, "--ep-dir")) ep_dir = v;
    else if (!strcmp(a, "--out")) out_path = v;
    else { fprintf(stderr, "unknown option %s\n", a); return 2; }
    ++i;
  }
  int world = 1, rank = 0;
  if (ep_dir) {
    const char* w = getenv("WORLD_SIZE");
    const char* r = getenv("RANK");
    const char* lr = getenv("LOCAL_RANK");
    world = w ? atoi(w) : 1;
    rank = r ? atoi(r) : 0;
    device = lr ? atoi(lr) : rank;
    if (world < 1 || rank < 0 || rank >= world || batch % world) {
      fprintf(stderr, "--ep-dir: WORLD_SIZE %d / RANK %d, batch %d not a multiple of the ranks\n", world, rank, batch);
      return 2;
    }
    batch /= world;                                 /* this rank's sequences */
    setenv("MOE_EP_WAIT_MS", "60000", 0);           /* ranks run host attention between calls */
  }
  if (moe_cuda_init(device, world, rank, NULL) != MOE_OK) {
    fprintf(stderr, "moe_cuda_init: %s\n", moe_cuda_last_error());
    return 1;
  }
  MhConfig cfg = {2048, layers, 128, 32, 4, 768, 128, 151936, 1000000.f, 1e-6f};
  if (bin) {
    if (mh_config_from_bin(bin, &cfg) != MOE_OK) { fprintf(stderr, "%s\n", mh_last_error()); return 1; }
    if (layers < cfg.n_layers) cfg.n_layers = layers;
  }
  const int need = kv_fill + prompt + steps;
  if (ctx < need) ctx = need;
  const double t_load = now_ms();
  MhModel* m = mh_create(&cfg, batch, ctx, 0);
  if (!m) { fprintf(stderr, "%s\n", mh_last_error()); return 1; }
  int rc = bin ? mh_load_bin(m, bin) : mh_synth(m, seed, dtype, 0.02f);
  if (rc) { fprintf(stderr, "weights: %s\n", mh_last_error()); mh_free(m); return 1; }
  const double load_ms = now_ms() - t_load;
  if (world > 1) {
    /* at most 256 routed tokens per call over all ranks (moe_ffn_ep) */
    int cap = 256 / world;
    if (cap > batch * prompt) cap = batch * prompt;
    unsigned char h[64], all[64 * 64];
    if (world > 64) { fprintf(stderr, "at most 64 ranks\n"); return 1; }
    if (mh_ep_setup(m, cap, h) || put_file(ep_dir, "handle", rank, h, 64) || wait_files(ep_dir, "handle", world)) {
      fprintf(stderr, "ep setup: %s\n", mh_last_error());
      return 1;
    }
    for (int r = 0; r < world; ++r) {
      char path[4096];
      snprintf(path, sizeof(path), "%s/handle.%d", ep_dir, r);
      FILE* f = fopen(path, "rb");
      if (!f || fread(all + 64 * r, 1, 64, f) != 64) { fprintf(stderr, "ep: read %s\n", path); return 1; }
      fclose(f);
    }
    if (mh_ep_connect(m, all) || barrier(ep_dir, "connected", rank, world)) {
      fprintf(stderr, "ep connect: %s\n", mh_last_error());
      return 1;
    }
  }

  int* prompts = (int*)malloc(sizeof(int) * (size_t)batch * prompt);
  int* out = (int*)malloc(sizeof(int) * (size_t)batch * steps);
  float* logits = (float*)malloc(sizeof(float) * (size_t)batch * cfg.vocab_size);
  /* the prompts of all ranks' sequences from one stream; this rank takes its rows */
  uint64_t s = seed ^ 0xA5A5A5A5ull;
  for (long i = 0; i < (long)batch * rank * prompt; ++i) splitmix(&s);
  for (int i = 0; i < batch * prompt; ++i) prompts[i] = (int)(splitmix(&s) % (uint64_t)cfg.vocab_size);

  /* prefill (prompt at position kv_fill), then steps-1 single-token steps */
  if (kv_fill && (rc = mh_fill_kv(m, kv_fill, seed + 17 + 1000003ull * rank, 1.0f))) {
    fprintf(stderr, "%s\n", mh_last_error());
    return 1;
  }
  if (!kv_fill) mh_reset(m);
  if (world > 1 && barrier(ep_dir, "start", rank, world)) return 1;
  mh_timing_reset(m);
  const double t0 = now_ms();
  rc = mh_step(m, prompts, prompt, logits);
  const double prefill_ms = now_ms() - t0;
  double pre_moe[1024] = {0}, pre_cpu = 0;
  long pre_calls[1024] = {0};
  if (cfg.n_layers > 1024) { fprintf(stderr, "too many layers\n"); return 1; }
  mh_timing(m, pre_moe, pre_calls, &pre_cpu);
  mh_timing_reset(m);
  int* ids = (int*)malloc(sizeof(int) * (size_t)batch);
  const double t1 = now_ms();
  for (int st = 0; !rc && st < steps; ++st) {
    mh_pick_greedy(m, logits, ids);
    for (int b = 0; b < batch; ++b) out[(size_t)b * steps + st] = ids[b];
    if (st + 1 < steps) rc = mh_step(m, ids, 1, logits);
  }
  const double decode_ms = now_ms() - t1;
  if (rc) { fprintf(stderr, "decode: %s\n", mh_last_error()); return 1; }
  if (world > 1 && barrier(ep_dir, "done", rank, world)) return 1;
  if (out_path) {
    char path[4096];
    snprintf(path, sizeof(path), "%s.%d", out_path, rank);
    FILE* f = fopen(path, "w");
    if (!f) { fprintf(stderr, "--out: %s: %s\n", path, strerror(errno)); return 1; }
    for (int b = 0; b < batch; ++b) {
      for (int st = 0; st < steps; ++st) fprintf(f, st ? " %d" : "%d", out[(size_t)b * steps + st]);
      fputc('\n', f);
    }
    fclose(f);
  }
  double* moe_ms = (double*)calloc((size_t)cfg.n_layers, sizeof(double));
  long* calls = (long*)calloc((size_t)cfg.n_layers, sizeof(long));
  double cpu_ms = 0, moe_total = 0;
  long call_total = 0;
  mh_timing(m, moe_ms, calls, &cpu_ms);
  for (int l = 0; l < cfg.n_layers; ++l) { moe_total += moe_ms[l]; call_total += calls[l]; }
  const int dsteps = steps - 1;
  if (rank == 0)
  printf("{\"workload\": \"greedy decode\", \"source\": \"%s\", \"layers\": %d, \"dtype\": \"%s\", "
         "\"ep_world\": %d, \"batch\": %d, \"prompt\": %d, \"steps\": %d, \"kv_fill\": %d, \"load_s\": %.2f, "
         "\"prefill_ms\": %.2f, \"decode_tok_s\": %.3f, \"decode_ms_per_step\": %.3f, "
         "\"moe_ms_per_layer_call\": %.4f, \"moe_ms_per_step\": %.3f, \"host_ms_per_step\": %.3f, "
         "\"first_tokens\": [%d, %d, %d, %d]}\n",
         bin ? "bin" : "synthetic", cfg.n_layers, dtype == MOE_DTYPE_Q8 ? "q8" : "q4", world, batch * world, prompt,
         steps, kv_fill, load_ms / 1e3, prefill_ms,
         dsteps > 0 ? (double)batch * world * dsteps / (decode_ms / 1e3) : 0.0,
         dsteps > 0 ? decode_ms / dsteps : 0.0, call_total ? moe_total / call_total : 0.0,
         dsteps > 0 ? moe_total / dsteps : 0.0, dsteps > 0 ? cpu_ms / dsteps : 0.0,
         out[0], steps > 1 ? out[1] : -1, steps > 2 ? out[2] : -1, steps > 3 ? out[3] : -1);
  free(moe_ms); free(calls); free(ids); free(prompts); free(out); free(logits);
  mh_free(m);
  moe_cuda_shutdown();
  return 0;
}
