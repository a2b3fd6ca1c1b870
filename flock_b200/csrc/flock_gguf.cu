// GGUF model files on the host, streamed into device planes.
//
// * The directory (web/js/gguf-dir.mjs:187 readDirectory, server/gguf.mjs:48
//   readModel): magic "GGUF", version 2 or 3, tensor and metadata counts,
//   typed metadata entries, tensor records (name, dims fastest-first, ggml
//   type, offset relative to the data section), data start = end of the
//   records rounded up to general.alignment (default 32).
// * The byte planner (gguf.mjs:78 byteRanges): absolute ranges covering a
//   layer span, merged across gaps of at most `gap` bytes.
// * The streaming repack (gguf-stream.mjs:132 SplitStreamer, :281
//   streamTensorToGPU): a tensor's bytes are read `staging` bytes at a time,
//   Q8_0 / Q4_0 blocks are de-interleaved into the qs and f16-scale planes as
//   they arrive (a block cut by a read boundary is carried to the next read),
//   and each filled staging buffer is copied to the device while the next one
//   fills (two pinned buffers, ordered by events on the device's stream), so
//   the host never holds more than two staging buffers of a tensor.
//
// GGUF shapes are [in, out]: shape[0] is the row width (cols) and the
// product of the remaining dims the row count.
#include <cuda_runtime.h>
#include <unistd.h>

#include <cstdio>

#include <algorithm>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "flock_internal.h"

using namespace flock;

namespace {

enum { G_F32 = 0, G_F16 = 1, G_Q4_0 = 2, G_Q8_0 = 8 };

// IEEE binary16 bits -> the same value as binary32 (every f16 is exact in f32):
// sign, 5-bit exponent (bias 15), 10-bit fraction; subnormals are frac * 2^-24.
float half_bits_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t ex = (h >> 10) & 0x1F, fr = h & 0x3FF;
  uint32_t bits;
  if (ex == 0x1F) {
    bits = sign | 0x7F800000u | (fr << 13);  // inf / nan
  } else if (ex == 0) {
    float v = (float)fr * (1.0f / 16777216.0f);  // exact: fr < 2^10, scale a power of two
    memcpy(&bits, &v, 4);
    bits |= sign;
  } else {
    bits = sign | ((ex + 112) << 23) | (fr << 13);  // rebias 15 -> 127
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// ggml block geometry (gguf-dir.mjs:24 BLOCK): {weights per block, bytes}
bool block_spec(int dtype, int64_t* block, int64_t* bytes) {
  static const struct { int t; int64_t b, n; } tab[] = {
      {0, 1, 4},     {1, 1, 2},     {2, 32, 18},   {3, 32, 20},   {6, 32, 22},
      {7, 32, 24},   {8, 32, 34},   {9, 32, 40},   {10, 256, 84}, {11, 256, 110},
      {12, 256, 144}, {13, 256, 176}, {14, 256, 210}, {15, 256, 292}};
  for (auto& e : tab)
    if (e.t == dtype) {
      *block = e.b;
      *bytes = e.n;
      return true;
    }
  return false;
}

struct MetaValue {
  int kind = 0;  // 0 int, 1 float, 2 string, 3 array
  int64_t i = 0;
  double f = 0.0;
  std::string s;
};

struct TensorRec {
  std::string name;
  std::vector<int64_t> shape;
  int dtype = 0;
  int64_t offset = 0, bytes = 0, rows = 1, cols = 1;
};

// A bounded reader over the file's header.
struct Reader {
  int fd = -1;
  int64_t at = 0, size = 0;
  bool ok = true;
  bool read(void* dst, int64_t n) {
    if (!ok || n < 0 || at + n > size) {
      ok = false;
      return false;
    }
    int64_t got = 0;
    while (got < n) {
      const ssize_t r = pread(fd, (char*)dst + got, (size_t)(n - got), (off_t)(at + got));
      if (r <= 0) {
        ok = false;
        return false;
      }
      got += r;
    }
    at += n;
    return true;
  }
  template <class T>
  T get() {
    T v{};
    read(&v, sizeof v);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > (uint64_t)(size - at)) {
      ok = false;
      return {};
    }
    std::string s((size_t)n, '\0');
    read(&s[0], (int64_t)n);
    return s;
  }
};

bool read_value(Reader& r, uint32_t type, MetaValue& v, int depth = 0) {
  switch (type) {
    case 0: v.i = r.get<uint8_t>(); break;
    case 1: v.i = r.get<int8_t>(); break;
    case 2: v.i = r.get<uint16_t>(); break;
    case 3: v.i = r.get<int16_t>(); break;
    case 4: v.i = r.get<uint32_t>(); break;
    case 5: v.i = r.get<int32_t>(); break;
    case 6: v.kind = 1; v.f = r.get<float>(); break;
    case 7: v.i = r.get<uint8_t>() != 0; break;
    case 8: v.kind = 2; v.s = r.str(); break;
    case 10: v.i = (int64_t)r.get<uint64_t>(); break;
    case 11: v.i = r.get<int64_t>(); break;
    case 12: v.kind = 1; v.f = r.get<double>(); break;
    case 9: {  // array: element type, count, elements (kept as a count)
      if (depth > 4) return false;
      const uint32_t et = r.get<uint32_t>();
      const uint64_t n = r.get<uint64_t>();
      v.kind = 3;
      v.i = (int64_t)n;
      for (uint64_t k = 0; k < n && r.ok; k++) {
        MetaValue e;
        if (!read_value(r, et, e, depth + 1)) return false;
      }
      break;
    }
    default: return false;
  }
  return r.ok;
}

}  // namespace

struct flock_gguf {
  FILE* f = nullptr;
  int fd = -1;
  int version = 0;
  int64_t file_size = 0, data_start = 0, alignment = 32;
  std::map<std::string, MetaValue> meta;
  std::vector<TensorRec> tensors;
  std::map<std::string, int64_t> by_name;
};

namespace {

const TensorRec* find_tensor(const flock_gguf* g, const char* name) {
  if (!g || !name) return nullptr;
  auto it = g->by_name.find(name);
  return it == g->by_name.end() ? nullptr : &g->tensors[(size_t)it->second];
}

// gguf-stream.mjs:132 SplitStreamer: whole blocks go to the planes, a block
// cut by a chunk boundary waits in `partial`; `flush` receives block-ordered
// runs of whole rows (qs bytes, scale bytes, first block index, block count).
struct SplitStreamer {
  int64_t bytes, qs_per_block, blocks_per_flush;
  std::vector<uint8_t> partial;
  int64_t partial_len = 0, pending = 0, emitted = 0;
  uint8_t* qs_out;
  uint8_t* sc_out;
  // returns a FLOCK_* status; may swap qs_out / sc_out (double buffering)
  int (*flush)(void* ctx, int64_t first_block, int64_t n_blocks);
  void* ctx;

  int block(const uint8_t* src) {
    sc_out[pending * 2] = src[0];
    sc_out[pending * 2 + 1] = src[1];
    memcpy(qs_out + pending * qs_per_block, src + 2, (size_t)qs_per_block);
    if (++pending == blocks_per_flush) return emit();
    return FLOCK_OK;
  }
  int emit() {
    if (!pending) return FLOCK_OK;
    const int rc = flush(ctx, emitted, pending);
    emitted += pending;
    pending = 0;
    return rc;
  }
  int push(const uint8_t* chunk, int64_t n) {
    int64_t at = 0;
    if (partial_len) {
      const int64_t want = std::min(bytes - partial_len, n);
      memcpy(partial.data() + partial_len, chunk, (size_t)want);
      partial_len += want;
      at = want;
      if (partial_len < bytes) return FLOCK_OK;
      FLOCK_TRY(block(partial.data()));
      partial_len = 0;
    }
    while (at + bytes <= n) {
      FLOCK_TRY(block(chunk + at));
      at += bytes;
    }
    if (n > at) {
      memcpy(partial.data(), chunk + at, (size_t)(n - at));
      partial_len = n - at;
    }
    return FLOCK_OK;
  }
  int end() {
    if (partial_len) {
      set_error("tensor ended mid-block: %lld of %lld bytes (a short read or the wrong range)",
                (long long)partial_len, (long long)bytes);
      return FLOCK_E_ARG;
    }
    return emit();
  }
};

// Feed [abs, abs + n) of the file through `push` in `chunk`-byte reads.
template <class Push>
int read_range(int fd, int64_t abs, int64_t n, int64_t chunk, std::vector<uint8_t>& buf,
               Push push) {
  buf.resize((size_t)std::min(chunk, n > 0 ? n : 1));
  int64_t done = 0;
  while (done < n) {
    const int64_t want = std::min((int64_t)buf.size(), n - done);
    int64_t got = 0;
    while (got < want) {
      const ssize_t r = pread(fd, buf.data() + got, (size_t)(want - got), (off_t)(abs + done + got));
      if (r <= 0) {
        set_error("short read at byte %lld of the file", (long long)(abs + done + got));
        return FLOCK_E_ARG;
      }
      got += r;
    }
    FLOCK_TRY(push(buf.data(), want));
    done += want;
  }
  return FLOCK_OK;
}

int quant_check(const TensorRec* t, const char* name) {
  if (!t) {
    set_error("no tensor named %s", name ? name : "(null)");
    return FLOCK_E_MISSING;
  }
  if (t->dtype != G_Q8_0 && t->dtype != G_Q4_0) {
    set_error("%s: ggml type %d is neither Q8_0 nor Q4_0", t->name.c_str(), t->dtype);
    return FLOCK_E_UNSUPPORTED;
  }
  if (t->cols % 32) {
    set_error("%s: %lld cols not divisible by 32", t->name.c_str(), (long long)t->cols);
    return FLOCK_E_ARG;
  }
  return FLOCK_OK;
}

// Device sink: two pinned staging pairs; each flush (whole rows) goes out by
// async copies on the device stream, the scales into the tensor's padded rows.
struct DeviceSink {
  flock_tensor* t;
  cudaStream_t st;
  uint8_t* qs_h[2] = {};
  uint8_t* sc_h[2] = {};
  cudaEvent_t ev[2] = {};
  int cur = 0;
  int64_t nb = 0, qs_per_block = 0;
  SplitStreamer* s = nullptr;

  static int flush(void* ctx, int64_t first, int64_t n) {
    DeviceSink* d = (DeviceSink*)ctx;
    const int64_t row0 = first / d->nb, rows = n / d->nb;
    FLOCK_CK(cudaMemcpyAsync(d->t->qs.as<uint8_t>() + first * d->qs_per_block, d->qs_h[d->cur],
                             (size_t)(n * d->qs_per_block), cudaMemcpyHostToDevice, d->st));
    FLOCK_CK(cudaMemcpy2DAsync(d->t->sc.as<uint8_t>() + row0 * d->t->sc_stride * 2,
                               (size_t)d->t->sc_stride * 2, d->sc_h[d->cur], (size_t)d->nb * 2,
                               (size_t)d->nb * 2, (size_t)rows, cudaMemcpyHostToDevice, d->st));
    FLOCK_CK(cudaEventRecord(d->ev[d->cur], d->st));
    // the other pair was handed to the copy engine one flush ago: wait for it
    d->cur ^= 1;
    FLOCK_CK(cudaEventSynchronize(d->ev[d->cur]));
    d->s->qs_out = d->qs_h[d->cur];
    d->s->sc_out = d->sc_h[d->cur];
    return FLOCK_OK;
  }
};

struct HostSink {
  uint8_t* qs;
  uint8_t* sc;
  int64_t qs_per_block;
  SplitStreamer* s;
  static int flush(void* ctx, int64_t first, int64_t n) {
    HostSink* h = (HostSink*)ctx;
    // the streamer wrote straight into the caller's planes; move its window on
    h->s->qs_out = h->qs + (first + n) * h->qs_per_block;
    h->s->sc_out = h->sc + (first + n) * 2;
    return FLOCK_OK;
  }
};

}  // namespace

extern "C" {

int flock_gguf_open(const char* path, flock_gguf** out) {
  if (!path || !out) return FLOCK_E_ARG;
  FILE* f = fopen(path, "rb");
  if (!f) {
    set_error("cannot open %s", path);
    return FLOCK_E_ARG;
  }
  flock_gguf* g = new flock_gguf();
  g->f = f;
  g->fd = fileno(f);
  const int fd = g->fd;
  g->file_size = (int64_t)lseek(fd, 0, SEEK_END);
  Reader r;
  r.fd = fd;
  r.size = g->file_size;
  auto fail = [&](const char* why) {
    set_error("%s: %s", path, why);
    flock_gguf_free(g);
    return FLOCK_E_ARG;
  };
  if (r.get<uint32_t>() != 0x46554747u) return fail("not a GGUF file");
  g->version = (int)r.get<uint32_t>();
  if (g->version != 2 && g->version != 3) return fail("unsupported GGUF version");
  const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
  if (!r.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) return fail("bad header counts");
  for (uint64_t i = 0; i < n_kv; i++) {
    const std::string key = r.str();
    const uint32_t type = r.get<uint32_t>();
    MetaValue v;
    if (!r.ok || !read_value(r, type, v)) return fail("bad metadata entry");
    g->meta[key] = v;
  }
  for (uint64_t i = 0; i < n_tensors; i++) {
    TensorRec t;
    t.name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    if (!r.ok || nd < 1 || nd > 4) return fail("bad tensor record");
    int64_t n = 1;
    for (uint32_t d = 0; d < nd; d++) {
      t.shape.push_back((int64_t)r.get<uint64_t>());
      if (t.shape.back() < 0 || t.shape.back() > ((int64_t)1 << 40)) return fail("bad tensor dims");
      n *= t.shape.back();
    }
    t.dtype = (int)r.get<uint32_t>();
    t.offset = (int64_t)r.get<uint64_t>();
    if (!r.ok) return fail("truncated tensor record");
    t.cols = t.shape[0];
    t.rows = n / (t.cols > 0 ? t.cols : 1);
    int64_t blk = 0, bb = 0;
    if (!block_spec(t.dtype, &blk, &bb) || n % blk) t.bytes = -1;  // not loadable
    else t.bytes = n / blk * bb;
    g->by_name[t.name] = (int64_t)g->tensors.size();
    g->tensors.push_back(t);
  }
  auto al = g->meta.find("general.alignment");
  if (al != g->meta.end() && al->second.kind == 0 && al->second.i > 0) g->alignment = al->second.i;
  g->data_start = (r.at + g->alignment - 1) / g->alignment * g->alignment;
  for (auto& t : g->tensors)
    if (t.bytes >= 0 && g->data_start + t.offset + t.bytes > g->file_size)
      return fail("a tensor runs past the end of the file");
  *out = g;
  return FLOCK_OK;
}

int flock_gguf_free(flock_gguf* g) {
  if (g) {
    if (g->f) fclose(g->f);
    delete g;
  }
  return FLOCK_OK;
}

int flock_gguf_info(const flock_gguf* g, int64_t* n_tensors, int64_t* data_start, int* version,
                    int* n_layers) {
  if (!g) return FLOCK_E_ARG;
  if (n_tensors) *n_tensors = (int64_t)g->tensors.size();
  if (data_start) *data_start = g->data_start;
  if (version) *version = g->version;
  if (n_layers) {
    *n_layers = -1;
    auto a = g->meta.find("general.architecture");
    if (a != g->meta.end() && a->second.kind == 2) {
      auto b = g->meta.find(a->second.s + ".block_count");
      if (b != g->meta.end() && b->second.kind == 0) *n_layers = (int)b->second.i;
    }
  }
  return FLOCK_OK;
}

int flock_gguf_tensor_info(const flock_gguf* g, int64_t i, char* name, int name_cap, int* dtype,
                           int64_t* rows, int64_t* cols, int64_t* offset, int64_t* bytes) {
  if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return FLOCK_E_ARG;
  const TensorRec& t = g->tensors[(size_t)i];
  if (name && name_cap > 0) {
    strncpy(name, t.name.c_str(), (size_t)name_cap - 1);
    name[name_cap - 1] = '\0';
  }
  if (dtype) *dtype = t.dtype;
  if (rows) *rows = t.rows;
  if (cols) *cols = t.cols;
  if (offset) *offset = t.offset;
  if (bytes) *bytes = t.bytes;
  return FLOCK_OK;
}

int flock_gguf_find(const flock_gguf* g, const char* name, int64_t* index) {
  if (!g || !name || !index) return FLOCK_E_ARG;
  auto it = g->by_name.find(name);
  if (it == g->by_name.end()) {
    set_error("no tensor named %s", name);
    return FLOCK_E_MISSING;
  }
  *index = it->second;
  return FLOCK_OK;
}

static const MetaValue* meta_of(const flock_gguf* g, const char* key) {
  if (!g || !key) return nullptr;
  auto it = g->meta.find(key);
  if (it == g->meta.end()) {
    set_error("no metadata key %s", key);
    return nullptr;
  }
  return &it->second;
}

int flock_gguf_meta_int(const flock_gguf* g, const char* key, int64_t* out) {
  const MetaValue* v = meta_of(g, key);
  if (!v || !out) return v ? FLOCK_E_ARG : FLOCK_E_MISSING;
  if (v->kind != 0 && v->kind != 3) return FLOCK_E_ARG;
  *out = v->i;  // arrays report their length
  return FLOCK_OK;
}

int flock_gguf_meta_f64(const flock_gguf* g, const char* key, double* out) {
  const MetaValue* v = meta_of(g, key);
  if (!v || !out) return v ? FLOCK_E_ARG : FLOCK_E_MISSING;
  if (v->kind == 1) *out = v->f;
  else if (v->kind == 0) *out = (double)v->i;
  else return FLOCK_E_ARG;
  return FLOCK_OK;
}

int flock_gguf_meta_str(const flock_gguf* g, const char* key, char* out, int cap) {
  const MetaValue* v = meta_of(g, key);
  if (!v || !out || cap < 1) return v ? FLOCK_E_ARG : FLOCK_E_MISSING;
  if (v->kind != 2) return FLOCK_E_ARG;
  strncpy(out, v->s.c_str(), (size_t)cap - 1);
  out[cap - 1] = '\0';
  return FLOCK_OK;
}

// server/gguf.mjs:78 byteRanges over the blk.<first..last>.* tensors.
int flock_gguf_layer_ranges(const flock_gguf* g, int first, int last, int64_t gap,
                            int64_t* starts, int64_t* ends, int cap, int* n) {
  if (!g || !n || first > last || gap < 0) return FLOCK_E_ARG;
  std::vector<std::pair<int64_t, int64_t>> ts;
  for (int l = first; l <= last; l++) {
    const std::string prefix = "blk." + std::to_string(l) + ".";
    for (auto& t : g->tensors)
      if (t.name.compare(0, prefix.size(), prefix) == 0 && t.bytes >= 0)
        ts.push_back({g->data_start + t.offset, g->data_start + t.offset + t.bytes});
  }
  std::sort(ts.begin(), ts.end());
  std::vector<std::pair<int64_t, int64_t>> out;
  for (auto& r : ts) {
    if (!out.empty() && r.first - out.back().second <= gap)
      out.back().second = std::max(out.back().second, r.second);
    else
      out.push_back(r);
  }
  *n = (int)out.size();
  if (!starts || !ends || cap < (int)out.size()) return out.empty() ? FLOCK_OK : FLOCK_E_LIMIT;
  for (size_t i = 0; i < out.size(); i++) {
    starts[i] = out[i].first;
    ends[i] = out[i].second;
  }
  return FLOCK_OK;
}

int flock_gguf_split_host(const flock_gguf* g, const char* name, int64_t chunk, uint8_t* qs,
                          uint8_t* scales) {
  const TensorRec* t = find_tensor(g, name);
  FLOCK_TRY(quant_check(t, name));
  if (!qs || !scales || chunk < 1) return FLOCK_E_ARG;
  SplitStreamer s;
  s.bytes = t->dtype == G_Q8_0 ? 34 : 18;
  s.qs_per_block = s.bytes - 2;
  s.blocks_per_flush = 1 << 16;
  s.partial.assign((size_t)s.bytes, 0);
  s.qs_out = qs;
  s.sc_out = scales;
  HostSink h{qs, scales, s.qs_per_block, &s};
  s.flush = HostSink::flush;
  s.ctx = &h;
  // host sink: blocks land in the caller's planes directly; the window moves per flush
  std::vector<uint8_t> buf;
  FLOCK_TRY(read_range(g->fd, g->data_start + t->offset, t->bytes, chunk, buf,
                       [&](const uint8_t* p, int64_t n) { return s.push(p, n); }));
  return s.end();
}

int flock_gguf_load_tensor(flock_dev* dev, const flock_gguf* g, const char* name, int64_t staging,
                           flock_tensor** out) {
  if (!dev || !g || !name || !out) return FLOCK_E_ARG;
  const TensorRec* t = find_tensor(g, name);
  if (!t) {
    set_error("no tensor named %s", name);
    return FLOCK_E_MISSING;
  }
  if (staging <= 0) staging = 4 << 20;  // gguf-stream.mjs:45 STAGING
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  std::vector<uint8_t> buf;
  if (t->dtype == G_F32 || t->dtype == G_F16) {
    // norm gains: a few KB, no split; f16 is widened exactly to f32
    const int64_t n = t->rows * t->cols;
    std::vector<float> f((size_t)n);
    int64_t at = 0;
    FLOCK_TRY(read_range(g->fd, g->data_start + t->offset, t->bytes, staging, buf,
                         [&](const uint8_t* p, int64_t nb) {
                           if (t->dtype == G_F32) {
                             memcpy((uint8_t*)f.data() + at, p, (size_t)nb);
                           } else {
                             for (int64_t k = 0; k + 1 < nb; k += 2) {
                               uint16_t h;
                               memcpy(&h, p + k, 2);
                               f[(size_t)((at + k) / 2)] = half_bits_to_float(h);
                             }
                           }
                           at += nb;
                           return FLOCK_OK;
                         }));
    return flock_tensor_from_f32(dev, f.data(), n, out);
  }
  FLOCK_TRY(quant_check(t, name));
  flock_tensor* T = new flock_tensor();
  T->dev = dev_retain(dev);
  T->dtype = t->dtype == G_Q8_0 ? FLOCK_Q8_0 : FLOCK_Q4_0;
  T->rows = t->rows;
  T->cols = t->cols;
  const int64_t nb = t->cols / 32;
  T->sc_stride = (int)((nb + 7) / 8 * 8);
  SplitStreamer s;
  s.bytes = t->dtype == G_Q8_0 ? 34 : 18;
  s.qs_per_block = s.bytes - 2;
  // whole rows per flush, about `staging` bytes of blocks
  const int64_t rows_per_flush = std::max<int64_t>(1, staging / (nb * s.bytes));
  s.blocks_per_flush = rows_per_flush * nb;
  s.partial.assign((size_t)s.bytes, 0);
  DeviceSink d;
  d.t = T;
  d.st = dev->stream;
  d.nb = nb;
  d.qs_per_block = s.qs_per_block;
  d.s = &s;
  int rc = FLOCK_OK;
  auto cleanup = [&]() {
    cudaStreamSynchronize(dev->stream);
    for (int k = 0; k < 2; k++) {
      if (d.qs_h[k]) cudaFreeHost(d.qs_h[k]);
      if (d.sc_h[k]) cudaFreeHost(d.sc_h[k]);
      if (d.ev[k]) cudaEventDestroy(d.ev[k]);
    }
  };
  if ((rc = T->qs.alloc((size_t)(t->rows * nb * s.qs_per_block))) ||
      (rc = T->sc.alloc((size_t)(t->rows * T->sc_stride * 2)))) {
    cleanup();
    flock_tensor_free(T);
    return rc;
  }
  cudaError_t e = cudaMemsetAsync(T->sc.p, 0, T->sc.bytes, dev->stream);
  for (int k = 0; k < 2 && e == cudaSuccess; k++) {
    e = cudaHostAlloc((void**)&d.qs_h[k], (size_t)(s.blocks_per_flush * s.qs_per_block),
                      cudaHostAllocDefault);
    if (e == cudaSuccess)
      e = cudaHostAlloc((void**)&d.sc_h[k], (size_t)(s.blocks_per_flush * 2), cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&d.ev[k], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(d.ev[k], dev->stream);
  }
  if (e != cudaSuccess) {
    set_error("staging for %s: %s", name, cudaGetErrorString(e));
    cleanup();
    flock_tensor_free(T);
    return FLOCK_E_CUDA;
  }
  s.qs_out = d.qs_h[0];
  s.sc_out = d.sc_h[0];
  s.flush = DeviceSink::flush;
  s.ctx = &d;
  rc = read_range(g->fd, g->data_start + t->offset, t->bytes, staging, buf,
                  [&](const uint8_t* p, int64_t n) { return s.push(p, n); });
  if (!rc) rc = s.end();
  if (!rc && cudaStreamSynchronize(dev->stream) != cudaSuccess) {
    set_error("upload of %s failed", name);
    rc = FLOCK_E_CUDA;
  }
  cleanup();
  if (rc) {
    flock_tensor_free(T);
    return rc;
  }
  *out = T;
  return FLOCK_OK;
}

}  // extern "C"
