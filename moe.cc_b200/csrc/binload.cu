// binload.cu — one MoE layer read from the reference's .bin weight file
// straight into device residency.
//
// File format (writer: export.py _save_tensor, :8-21; reader: io.c:193-285):
//   6-byte magic "QW3W\0\1", a u32 tensor count (informational: the reader
//   goes on to end of file), then records
//     u32 name_len | name bytes | u32 dtype (0 f32, 1 f16, 2 i8, 3 u8 packed
//     int4) | u32 ndim | u32 shape[ndim] | data (elems x 4/2/1/1 bytes)
//   all little-endian.
// Tensor names of one layer L (model.h:212-305):
//   model.layers.L.mlp.gate.weight            f32 [E, D] (or mlp.router.gate.weight)
//   model.layers.L.mlp.gate.bias              f32 [E]    optional
//   model.layers.L.mlp.experts.e.{gate,up,down}_proj.weight.{q8|q4}
//   model.layers.L.mlp.experts.e.{gate,up,down}_proj.weight.scale  f32 [rows]
// Q4 tensors hold shape [rows, cols/2]; the logical cols are twice the
// stored ones (model.h:262). E is the number of consecutive experts present
// from 0 (model.h:133-155), and a repeated name resolves to its first record
// (io.c:333-338, a linear search).
//
// Unlike the reference's loader, which mallocs and reads every tensor of the
// file, this one walks the record headers once (seeking past the data) into a
// name index, then reads only the requested layer's router and this rank's
// experts, each straight into a pinned slab image whose host-to-device copy
// overlaps the read of the next expert. Malformed files
// and missing tensors return MOE_ERR_INVALID with a message where the
// reference exits the process.
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/moe_cuda.h"
#include "kernels.cuh"

namespace moe {
int set_error_message(int code, const char* msg);                       // runtime.cu
int upload_layer_streamed(int layer, const QuantizedWeight* Wg, const QuantizedWeight* Wu,
                          const QuantizedWeight* Wd, const float* router_w, const float* router_b, int E,
                          const ExpertReader& reader);                    // runtime.cu

namespace {

struct Rec {
  int dtype = 0, ndim = 0;
  uint32_t shape[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  uint64_t off = 0, bytes = 0;   // data position in the file and its size
};

struct BinIndex {
  std::unordered_map<std::string, Rec> recs;
  const Rec* find(const std::string& k) const {
    auto it = recs.find(k);
    return it == recs.end() ? nullptr : &it->second;
  }
};

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return set_error_message(code, buf);
}

bool rd_u32(FILE* f, uint32_t* v) { return fread(v, 4, 1, f) == 1; }

// Walks every record header of the file into `ix`.
int index_file(const char* path, FILE* f, BinIndex& ix) {
  struct stat st;
  if (fstat(fileno(f), &st) != 0) return fail(MOE_ERR_INVALID, "%s: cannot stat", path);
  const uint64_t fsize = (uint64_t)st.st_size;
  unsigned char magic[6];
  static const unsigned char want[6] = {'Q', 'W', '3', 'W', 0x00, 0x01};
  uint32_t count = 0;
  if (fread(magic, 1, 6, f) != 6 || memcmp(magic, want, 6) != 0)
    return fail(MOE_ERR_INVALID, "%s: bad magic (not a QW3W v1 weight file)", path);
  if (!rd_u32(f, &count)) return fail(MOE_ERR_INVALID, "%s: truncated header", path);
  std::string name;
  for (;;) {
    uint32_t nlen;
    if (!rd_u32(f, &nlen)) break;                       // end of file
    if (nlen == 0 || nlen > 4096) return fail(MOE_ERR_INVALID, "%s: bad name length %u", path, nlen);
    name.resize(nlen);
    if (fread(&name[0], 1, nlen, f) != nlen) return fail(MOE_ERR_INVALID, "%s: truncated name", path);
    uint32_t dt, nd;
    if (!rd_u32(f, &dt) || !rd_u32(f, &nd))
      return fail(MOE_ERR_INVALID, "%s: truncated header of %s", path, name.c_str());
    if (dt > 3) return fail(MOE_ERR_INVALID, "%s: %s has unknown dtype %u", path, name.c_str(), dt);
    if (nd > 8) return fail(MOE_ERR_INVALID, "%s: %s has %u dimensions", path, name.c_str(), nd);
    Rec r;
    r.dtype = (int)dt; r.ndim = (int)nd;
    uint64_t elems = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      uint32_t v;
      if (!rd_u32(f, &v)) return fail(MOE_ERR_INVALID, "%s: truncated shape of %s", path, name.c_str());
      r.shape[d] = v;
      elems *= v;
      if (elems > fsize) return fail(MOE_ERR_INVALID, "%s: %s is larger than the file", path, name.c_str());
    }
    r.bytes = elems * (dt == 0 ? 4 : dt == 1 ? 2 : 1);
    const long pos = ftell(f);
    if (pos < 0) return fail(MOE_ERR_INVALID, "%s: ftell failed", path);
    r.off = (uint64_t)pos;
    if (r.off + r.bytes > fsize) return fail(MOE_ERR_INVALID, "%s: %s is truncated", path, name.c_str());
    if (fseeko(f, (off_t)r.bytes, SEEK_CUR) != 0) return fail(MOE_ERR_INVALID, "%s: seek failed", path);
    ix.recs.emplace(name, r);                           // first record of a name wins
  }
  return MOE_OK;
}

// One layer's tensors, checked for shape and dtype.
struct LayerRecs {
  int E = 0, D = 0, F = 0, dtype = 0;
  const Rec* router = nullptr;
  const Rec* bias = nullptr;
  std::vector<const Rec*> q[3], s[3];   // gate, up, down
};

const char* const kProj[3] = {"gate_proj", "up_proj", "down_proj"};

std::string expert_key(int L, int e, int p, const char* suffix) {
  char k[256];
  snprintf(k, sizeof(k), "model.layers.%d.mlp.experts.%d.%s.weight.%s", L, e, kProj[p], suffix);
  return k;
}

int resolve_layer(const char* path, const BinIndex& ix, int L, LayerRecs& lr) {
  char k[256];
  snprintf(k, sizeof(k), "model.layers.%d.mlp.gate.weight", L);
  lr.router = ix.find(k);
  if (!lr.router) {
    snprintf(k, sizeof(k), "model.layers.%d.mlp.router.gate.weight", L);
    lr.router = ix.find(k);
  }
  if (!lr.router) return fail(MOE_ERR_INVALID, "%s: layer %d has no router (mlp.gate.weight)", path, L);
  snprintf(k, sizeof(k), "model.layers.%d.mlp.gate.bias", L);
  lr.bias = ix.find(k);
  if (lr.bias && lr.bias->dtype != 0) lr.bias = nullptr;   // only an f32 bias is used (model.h:218)

  const bool q8 = ix.find(expert_key(L, 0, 0, "q8")) != nullptr;
  const bool q4 = !q8 && ix.find(expert_key(L, 0, 0, "q4")) != nullptr;
  if (!q8 && !q4) {
    snprintf(k, sizeof(k), "model.layers.%d.mlp.experts.0.gate_proj.weight", L);
    if (ix.find(k))
      return fail(MOE_ERR_UNSUPPORTED, "%s: layer %d experts are not quantised (export with --quant q8 or q4)",
                  path, L);
    return fail(MOE_ERR_INVALID, "%s: layer %d has no experts", path, L);
  }
  const char* qs = q8 ? "q8" : "q4";
  lr.dtype = q8 ? MOE_DTYPE_Q8 : MOE_DTYPE_Q4;
  // E: consecutive experts from 0 whose down projection exists (model.h:133-155)
  while (ix.find(expert_key(L, lr.E, 2, qs))) ++lr.E;
  if (lr.E == 0) return fail(MOE_ERR_INVALID, "%s: layer %d has no expert 0 down_proj", path, L);
  const Rec* g0 = ix.find(expert_key(L, 0, 0, qs));
  if (g0->ndim != 2) return fail(MOE_ERR_INVALID, "%s: layer %d gate_proj is not 2-D", path, L);
  lr.F = (int)g0->shape[0];
  lr.D = (int)g0->shape[1] * (q4 ? 2 : 1);
  for (int p = 0; p < 3; ++p) { lr.q[p].resize(lr.E); lr.s[p].resize(lr.E); }
  for (int e = 0; e < lr.E; ++e) {
    for (int p = 0; p < 3; ++p) {
      const std::string kq = expert_key(L, e, p, qs), ks = expert_key(L, e, p, "scale");
      const Rec* rq = ix.find(kq);
      const Rec* rs = ix.find(ks);
      if (!rq) return fail(MOE_ERR_INVALID, "%s: missing %s", path, kq.c_str());
      if (!rs) return fail(MOE_ERR_INVALID, "%s: missing %s", path, ks.c_str());
      const uint32_t rows = p < 2 ? lr.F : lr.D, cols = p < 2 ? lr.D : lr.F;
      const uint32_t stored = q4 ? cols / 2 : cols;
      if (rq->dtype != (q8 ? 2 : 3) || rq->ndim != 2 || rq->shape[0] != rows || rq->shape[1] != stored)
        return fail(MOE_ERR_INVALID, "%s: %s has dtype %d shape [%u,%u], expected [%u,%u]", path, kq.c_str(),
                    rq->dtype, rq->shape[0], rq->ndim > 1 ? rq->shape[1] : 0, rows, stored);
      if (rs->dtype != 0 || rs->bytes != 4ull * rows)
        return fail(MOE_ERR_INVALID, "%s: %s is not f32 [%u]", path, ks.c_str(), rows);
      lr.q[p][e] = rq; lr.s[p][e] = rs;
    }
  }
  if (lr.router->dtype != 0 || lr.router->bytes != 4ull * lr.E * lr.D)
    return fail(MOE_ERR_INVALID, "%s: layer %d router is not f32 [%d,%d]", path, L, lr.E, lr.D);
  if (lr.bias && lr.bias->bytes != 4ull * lr.E) lr.bias = nullptr;
  return MOE_OK;
}

bool read_at(FILE* f, const Rec* r, void* dst) {
  return fseeko(f, (off_t)r->off, SEEK_SET) == 0 && fread(dst, 1, r->bytes, f) == r->bytes;
}

}  // namespace

// An open weight file: the FILE and its name index (bin_load + bin_find of
// io.c:193-338, without reading the data).
struct BinHandle {
  FILE* f = nullptr;
  std::string path;
  BinIndex ix;
  std::mutex mu;   // one reader at a time on the FILE position
  ~BinHandle() { if (f) fclose(f); }
};

}  // namespace moe

using namespace moe;
struct MoeBin : BinHandle {};

extern "C" {

MoeBin* moe_bin_open(const char* path) {
  if (!path) { fail(MOE_ERR_INVALID, "path is NULL"); return nullptr; }
  MoeBin* h = new MoeBin;
  h->path = path;
  h->f = fopen(path, "rb");
  if (!h->f) { fail(MOE_ERR_INVALID, "%s: cannot open", path); delete h; return nullptr; }
  if (index_file(path, h->f, h->ix)) { delete h; return nullptr; }
  return h;
}

void moe_bin_close(MoeBin* h) { delete h; }

int moe_bin_find(MoeBin* h, const char* name, int* dtype, int* ndim, int* shape, size_t* nbytes) {
  if (!h || !name) return fail(MOE_ERR_INVALID, "moe_bin_find: NULL handle or name");
  const Rec* r = h->ix.find(name);
  if (!r) return fail(MOE_ERR_INVALID, "%s: missing %s", h->path.c_str(), name);
  if (dtype) *dtype = r->dtype;
  if (ndim) *ndim = r->ndim;
  if (shape) for (int d = 0; d < r->ndim; ++d) shape[d] = (int)r->shape[d];
  if (nbytes) *nbytes = (size_t)r->bytes;
  return MOE_OK;
}

int moe_bin_read(MoeBin* h, const char* name, void* dst, size_t nbytes) {
  if (!h || !name || !dst) return fail(MOE_ERR_INVALID, "moe_bin_read: NULL argument");
  const Rec* r = h->ix.find(name);
  if (!r) return fail(MOE_ERR_INVALID, "%s: missing %s", h->path.c_str(), name);
  if (r->bytes != nbytes)
    return fail(MOE_ERR_INVALID, "%s: %s holds %llu bytes, not %zu", h->path.c_str(), name,
                (unsigned long long)r->bytes, nbytes);
  std::lock_guard<std::mutex> lk(h->mu);
  if (!read_at(h->f, r, dst)) return fail(MOE_ERR_INVALID, "%s: read of %s failed", h->path.c_str(), name);
  return MOE_OK;
}

int moe_bin_layer_info_h(MoeBin* h, int src_layer, int* E, int* D, int* F, int* dtype, int* has_bias) {
  if (!h) return fail(MOE_ERR_INVALID, "moe_bin_layer_info_h: NULL handle");
  LayerRecs lr;
  const int rc = resolve_layer(h->path.c_str(), h->ix, src_layer, lr);
  if (rc) return rc;
  if (E) *E = lr.E;
  if (D) *D = lr.D;
  if (F) *F = lr.F;
  if (dtype) *dtype = lr.dtype;
  if (has_bias) *has_bias = lr.bias != nullptr;
  return MOE_OK;
}

int moe_bin_layer_info(const char* path, int src_layer, int* E, int* D, int* F, int* dtype, int* has_bias) {
  MoeBin* h = moe_bin_open(path);
  if (!h) return MOE_ERR_INVALID;
  const int rc = moe_bin_layer_info_h(h, src_layer, E, D, F, dtype, has_bias);
  moe_bin_close(h);
  return rc;
}

int moe_cuda_load_bin_layer_h(MoeBin* h, int src_layer, int layer) {
  if (!h) return fail(MOE_ERR_INVALID, "moe_cuda_load_bin_layer_h: NULL handle");
  struct Ctx {
    BinHandle* h;
    LayerRecs lr;
  } c;
  c.h = h;
  int rc = resolve_layer(h->path.c_str(), h->ix, src_layer, c.lr);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(h->mu);
  const LayerRecs& lr = c.lr;
  std::vector<unsigned char> router(lr.router->bytes + (lr.bias ? lr.bias->bytes : 0));
  if (!read_at(h->f, lr.router, router.data()) || (lr.bias && !read_at(h->f, lr.bias, router.data() + lr.router->bytes)))
    return fail(MOE_ERR_INVALID, "%s: read of the layer %d router failed", h->path.c_str(), src_layer);
  // the experts' q/s pointers are placeholders (shapes only): the slab
  // images come from `fill`, read straight into pinned staging
  static const float placeholder[1] = {0.0f};
  std::vector<QuantizedWeight> W[3];
  for (int p = 0; p < 3; ++p) {
    W[p].resize(lr.E);
    for (QuantizedWeight& w : W[p]) {
      w.rows = p < 2 ? lr.F : lr.D;
      w.cols = p < 2 ? lr.D : lr.F;
      w.dtype = lr.dtype;
      w.q = (const int8_t*)placeholder;
      w.s = placeholder;
    }
  }
  ExpertReader rd;
  rd.ctx = &c;
  rd.fill = [](void* ctx, int e, const LayerDev& L, uint8_t* img) -> bool {
    Ctx& c = *static_cast<Ctx*>(ctx);
    const size_t qoff[3] = {L.gq_off, L.uq_off, L.dq_off}, soff[3] = {L.gs_off, L.us_off, L.ds_off};
    for (int p = 0; p < 3; ++p)
      if (!read_at(c.h->f, c.lr.q[p][e], img + qoff[p]) || !read_at(c.h->f, c.lr.s[p][e], img + soff[p])) {
        fail(MOE_ERR_INVALID, "%s: read of expert %d failed", c.h->path.c_str(), e);
        return false;
      }
    return true;
  };
  return upload_layer_streamed(layer, W[0].data(), W[1].data(), W[2].data(), (const float*)router.data(),
                               lr.bias ? (const float*)(router.data() + lr.router->bytes) : nullptr, lr.E, rd);
}

int moe_cuda_load_bin_layer(const char* path, int src_layer, int layer) {
  MoeBin* h = moe_bin_open(path);
  if (!h) return MOE_ERR_INVALID;
  const int rc = moe_cuda_load_bin_layer_h(h, src_layer, layer);
  moe_bin_close(h);
  return rc;
}

}  // extern "C"
