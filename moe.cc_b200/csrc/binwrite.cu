// binwrite.cu — host-side writers of the .bin weight format and the rowwise
// quantisers on the host.
//
// The writer produces the layout of export.py's single-file mode and of
// merge_dir.py (export.py:188-206, merge_dir.py:34-43): magic "QW3W\0\1", a
// u32 count fixed when the file is created, then the records appended in
// order. merge_dir.py writes the number of ORIGINAL tensors as that count
// while a quantised tensor contributes two records (.scale, then .q8/.q4),
// so the count is the caller's to choose and is never patched; readers go to
// end of file (io.c:212-233).
//
// The host quantisers give export._rowwise_q8 / _rowwise_q4 (export.py:23-36)
// bit for bit, as the device ones do: s = max(max|row|, 1e-8) / 127 (or / 7)
// in fp32, q = round-half-even(w / s) with an IEEE divide; Q4 clamps to
// [-8, 7], adds 8 and packs the even column into the low nibble.
#include <fenv.h>
#include <math.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/moe_cuda.h"

namespace moe {
int set_error_message(int code, const char* msg);   // runtime.cu
namespace {
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return set_error_message(code, buf);
}

// max(max|row|, 1e-8) / S
float row_scale(const float* w, int cols, float S) {
  float amax = 0.0f;
  for (int c = 0; c < cols; ++c) {
    const float a = fabsf(w[c]);
    if (a > amax) amax = a;
  }
  if (amax < 1e-8f) amax = 1e-8f;   // clamp(min=1e-8), export.py:25,31
  return amax / S;
}
}  // namespace
}  // namespace moe

using namespace moe;

struct MoeBinWriter {
  FILE* f = nullptr;
  long long records = 0;
};

extern "C" {

MoeBinWriter* moe_bin_create(const char* path, uint32_t count) {
  if (!path) { fail(MOE_ERR_INVALID, "moe_bin_create: NULL path"); return nullptr; }
  FILE* f = fopen(path, "wb");
  if (!f) { fail(MOE_ERR_INVALID, "%s: cannot create", path); return nullptr; }
  static const unsigned char magic[6] = {'Q', 'W', '3', 'W', 0x00, 0x01};
  if (fwrite(magic, 1, 6, f) != 6 || fwrite(&count, 4, 1, f) != 1) {
    fclose(f);
    fail(MOE_ERR_INVALID, "%s: write failed", path);
    return nullptr;
  }
  MoeBinWriter* w = new MoeBinWriter;
  w->f = f;
  return w;
}

int moe_bin_put(MoeBinWriter* w, const char* name, int dtype, int ndim, const int* shape, const void* data) {
  if (!w || !w->f || !name || ndim < 0 || ndim > 8 || (ndim && !shape) || dtype < 0 || dtype > 3)
    return fail(MOE_ERR_INVALID, "moe_bin_put: bad argument");
  uint64_t elems = 1;
  for (int d = 0; d < ndim; ++d) {
    if (shape[d] < 0) return fail(MOE_ERR_INVALID, "moe_bin_put: negative extent in %s", name);
    elems *= (uint64_t)shape[d];
  }
  const uint64_t bytes = elems * (dtype == 0 ? 4 : dtype == 1 ? 2 : 1);
  if (bytes && !data) return fail(MOE_ERR_INVALID, "moe_bin_put: NULL data for %s", name);
  const uint32_t nlen = (uint32_t)strlen(name), dt = (uint32_t)dtype, nd = (uint32_t)ndim;
  uint32_t sh[8];
  for (int d = 0; d < ndim; ++d) sh[d] = (uint32_t)shape[d];
  if (fwrite(&nlen, 4, 1, w->f) != 1 || fwrite(name, 1, nlen, w->f) != nlen || fwrite(&dt, 4, 1, w->f) != 1 ||
      fwrite(&nd, 4, 1, w->f) != 1 || (nd && fwrite(sh, 4, nd, w->f) != nd) ||
      (bytes && fwrite(data, 1, bytes, w->f) != bytes))
    return fail(MOE_ERR_INVALID, "moe_bin_put: write of %s failed", name);
  w->records++;
  return MOE_OK;
}

int moe_bin_finish(MoeBinWriter* w) {
  if (!w) return fail(MOE_ERR_INVALID, "moe_bin_finish: NULL writer");
  const int bad = fclose(w->f) != 0;
  delete w;
  return bad ? fail(MOE_ERR_INVALID, "moe_bin_finish: close failed") : MOE_OK;
}

int moe_quantize_rowwise_q8_host(const float* W, int rows, int cols, int8_t* q, float* s) {
  if (!W || !q || !s || rows < 0 || cols < 1) return fail(MOE_ERR_INVALID, "moe_quantize_rowwise_q8_host: bad argument");
  if (fegetround() != FE_TONEAREST) return fail(MOE_ERR_INVALID, "quantiser needs round-to-nearest mode");
#pragma omp parallel for schedule(static) if (rows >= 64)
  for (int r = 0; r < rows; ++r) {
    const float* w = W + (size_t)r * cols;
    const float sc = row_scale(w, cols, 127.0f);
    s[r] = sc;
    for (int c = 0; c < cols; ++c) q[(size_t)r * cols + c] = (int8_t)(int)rintf(w[c] / sc);
  }
  return MOE_OK;
}

int moe_quantize_rowwise_q4_host(const float* W, int rows, int cols, uint8_t* q, float* s) {
  if (!W || !q || !s || rows < 0 || cols < 2 || (cols & 1))
    return fail(MOE_ERR_INVALID, "moe_quantize_rowwise_q4_host: bad argument (cols must be even)");
  if (fegetround() != FE_TONEAREST) return fail(MOE_ERR_INVALID, "quantiser needs round-to-nearest mode");
#pragma omp parallel for schedule(static) if (rows >= 64)
  for (int r = 0; r < rows; ++r) {
    const float* w = W + (size_t)r * cols;
    const float sc = row_scale(w, cols, 7.0f);
    s[r] = sc;
    uint8_t* qr = q + (size_t)r * (cols / 2);
    for (int c = 0; c < cols; c += 2) {
      float v0 = rintf(w[c] / sc), v1 = rintf(w[c + 1] / sc);
      v0 = v0 < -8.f ? -8.f : v0 > 7.f ? 7.f : v0;
      v1 = v1 < -8.f ? -8.f : v1 > 7.f ? 7.f : v1;
      qr[c / 2] = (uint8_t)(((int)v0 + 8) | (((int)v1 + 8) << 4));
    }
  }
  return MOE_OK;
}

}  // extern "C"
