// FLK1 frames (web/js/wire.mjs) at the C boundary, so a CUDA stage can sit in
// the reference's mesh: a coordinator or an upstream device sends
//   "FLK1" | seq u32 | hidden u32 | offset u32 | flags u32 | f16 payload
// and expects the same header back with the stage's output hidden state.
//
// * flock_wire_pack / flock_wire_unpack: the host codecs (wire.mjs:54 pack,
//   :79 unpack), f32 -> f16 rounding to nearest even with subnormals,
//   overflow to infinity and NaN as 0x7e00 | sign (wire.mjs:31 f32to16),
//   f16 -> f32 exactly with NaN canonical (wire.mjs:57 f16to32).
// * flock_range_forward_wire: web/bird.html:544 runFrame on the device -- the
//   f16 payload goes up as is (half the bytes of f32) and is widened by a
//   kernel into the first layer's input, the layers run in order (reset flag
//   clears their caches first; the frame's offset must equal the caches'
//   position), the last layer's output is rounded to f16 by a kernel with
//   the same rounding as f32to16 and only the f16 payload comes back.
// * flock_quant_q8 / flock_quant_q4: the host quantizers (kernels/lib.ts:40,
//   :64), which store their block scales with the same f16 rounding.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "flock_internal.h"

using namespace flock;

namespace {

constexpr uint32_t kMagic = 0x314b4c46;  // "FLK1" little-endian
constexpr uint32_t kFlagReset = 1, kFlagReplay = 2;

__host__ __device__ inline uint16_t f32_to_f16_rne(float v) {
  uint32_t x;
  memcpy(&x, &v, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  int e = (int)((x >> 23) & 0xff);
  uint32_t man = x & 0x7fffffu;
  if (e == 255) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));  // inf / nan
  e = e - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);  // overflow
  if (e <= 0) {  // subnormal (or zero)
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    const int shift = 14 - e;
    const uint32_t sub = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
    return (uint16_t)(sign | (sub + ((rem > half || (rem == half && (sub & 1u))) ? 1u : 0u)));
  }
  uint32_t h = ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1fffu;  // dropped bits
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;  // may carry into the exponent
  return (uint16_t)(sign | h);
}

__host__ __device__ inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  uint32_t bits;
  if (e == 31) {
    bits = man ? 0x7fc00000u : (sign | 0x7f800000u);  // NaN (canonical) / inf
  } else if (e == 0) {
    float v = (float)man * (1.0f / 16777216.0f);  // man * 2^-24, exact
    memcpy(&bits, &v, 4);
    bits |= sign;
  } else {
    bits = sign | ((e + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

__global__ void k_f16_to_f32(const uint16_t* __restrict__ in, float* __restrict__ out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = f16_to_f32(in[i]);
}
__global__ void k_f32_to_f16(const float* __restrict__ in, uint16_t* __restrict__ out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = f32_to_f16_rne(in[i]);
}

void put_u32(uint8_t* p, uint32_t v) { memcpy(p, &v, 4); }
uint32_t get_u32(const uint8_t* p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}

}  // namespace

extern "C" {

int flock_wire_pack(const float* x, int64_t n, uint32_t seq, uint32_t hidden, uint32_t offset,
                    uint32_t flags, uint8_t* out, int64_t cap, int64_t* out_len) {
  if (!x || n < 0 || !out || !out_len) return FLOCK_E_ARG;
  const int64_t need = 20 + 2 * n;
  *out_len = need;
  if (cap < need) {
    set_error("frame needs %lld bytes, buffer has %lld", (long long)need, (long long)cap);
    return FLOCK_E_LIMIT;
  }
  put_u32(out, kMagic);
  put_u32(out + 4, seq);
  put_u32(out + 8, hidden);
  put_u32(out + 12, offset);
  put_u32(out + 16, flags & (kFlagReset | kFlagReplay));
  for (int64_t i = 0; i < n; i++) {
    const uint16_t h = f32_to_f16_rne(x[i]);
    memcpy(out + 20 + 2 * i, &h, 2);
  }
  return FLOCK_OK;
}

int flock_wire_unpack(const uint8_t* frame, int64_t len, float* out, int64_t cap,
                      uint32_t meta[5]) {
  if (!frame || !meta || len < 20 || (len - 20) % 2) {
    set_error("not a flock frame (%lld bytes)", (long long)len);
    return FLOCK_E_ARG;
  }
  if (get_u32(frame) != kMagic) {
    set_error("not a flock frame");
    return FLOCK_E_ARG;
  }
  const int64_t n = (len - 20) / 2;
  const uint32_t flags = get_u32(frame + 16);
  meta[0] = get_u32(frame + 4);
  meta[1] = get_u32(frame + 8);
  meta[2] = get_u32(frame + 12);
  meta[3] = (flags & kFlagReset) ? 1u : 0u;
  meta[4] = (flags & kFlagReplay) ? 1u : 0u;
  if (!out) return FLOCK_OK;  // header only
  if (cap < n) return FLOCK_E_LIMIT;
  for (int64_t i = 0; i < n; i++) {
    uint16_t h;
    memcpy(&h, frame + 20 + 2 * i, 2);
    out[i] = f16_to_f32(h);
  }
  return FLOCK_OK;
}

int flock_range_forward_wire(flock_layer* const* layers, int n_layers, const uint8_t* frame,
                             int64_t frame_len, uint8_t* out, int64_t out_cap,
                             int64_t* out_len) {
  if (!layers || n_layers < 1 || !frame || !out || !out_len) return FLOCK_E_ARG;
  uint32_t meta[5];
  FLOCK_TRY(flock_wire_unpack(frame, frame_len, nullptr, 0, meta));
  const int seq = (int)meta[0], hidden = (int)meta[1], offset = (int)meta[2];
  const int64_t n = (frame_len - 20) / 2;
  for (int i = 0; i < n_layers; i++)
    if (!layers[i] || layers[i]->dev != layers[0]->dev ||
        layers[i]->cfg.hidden != layers[0]->cfg.hidden) {
      set_error("range_forward: layers must share one device and hidden size");
      return FLOCK_E_ARG;
    }
  if (hidden != layers[0]->cfg.hidden || seq < 1 || n != (int64_t)seq * hidden) {
    set_error("frame carries %lld values for seq %d x hidden %d; these layers take hidden %d",
              (long long)n, seq, hidden, layers[0]->cfg.hidden);
    return FLOCK_E_ARG;
  }
  *out_len = frame_len;
  if (out_cap < frame_len) {
    set_error("output frame needs %lld bytes, buffer has %lld", (long long)frame_len,
              (long long)out_cap);
    return FLOCK_E_LIMIT;
  }
  // bird.html:544 runFrame: a reset clears every held layer's cache first; the
  // frame must then start where the caches end
  for (int i = 0; i < n_layers; i++) {
    if (meta[3]) FLOCK_TRY(flock_layer_reset(layers[i]));
    if (layers[i]->n_keys != offset) {
      set_error("cache holds %d positions, frame is at %d", layers[i]->n_keys, offset);
      return FLOCK_E_STATE;
    }
  }
  flock_layer* first = layers[0];
  flock_layer* last = layers[n_layers - 1];
  if (seq > first->cfg.max_prefill) {
    set_error("prefill of %d exceeds maxPrefill %d; chunk it", seq, first->cfg.max_prefill);
    return FLOCK_E_STATE;
  }
  flock_dev* d = first->dev;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  Workspace* wi = first->ws;
  if (wi->wire.bytes < (size_t)n * 2) FLOCK_TRY(wi->wire.alloc((size_t)n * 2));
  FLOCK_CK(cudaMemcpyAsync(wi->wire.p, frame + 20, (size_t)n * 2, cudaMemcpyHostToDevice,
                           d->stream));
  const unsigned grid = (unsigned)((n + 255) / 256);
  k_f16_to_f32<<<grid, 256, 0, d->stream>>>(wi->wire.as<uint16_t>(), wi->h.as<float>(), n);
  FLOCK_CK(cudaGetLastError());
  FLOCK_TRY(flock_layer_encode(first, nullptr, seq));
  for (int i = 1; i < n_layers; i++) {
    if (layers[i]->ws != layers[i - 1]->ws)
      FLOCK_CK(cudaMemcpyAsync(layers[i]->ws->h.p, layers[i - 1]->ws->h.p, (size_t)n * 4,
                               cudaMemcpyDeviceToDevice, d->stream));
    FLOCK_TRY(flock_layer_encode(layers[i], nullptr, seq));
  }
  Workspace* wo = last->ws;
  if (wo->wire.bytes < (size_t)n * 2) FLOCK_TRY(wo->wire.alloc((size_t)n * 2));
  k_f32_to_f16<<<grid, 256, 0, d->stream>>>(wo->h.as<float>(), wo->wire.as<uint16_t>(), n);
  FLOCK_CK(cudaGetLastError());
  memcpy(out, frame, 20);  // the header travels on unchanged (flags included)
  FLOCK_CK(cudaMemcpyAsync(out + 20, wo->wire.p, (size_t)n * 2, cudaMemcpyDeviceToHost,
                           d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return ws_check_errors(wo);
}


// kernels/lib.ts:40 quantRowQ8 over every row.  JS numbers are f64: amax and
// d = amax/127 are f64, the stored scale is f32(d) rounded to f16 nearest-even
// (wire.mjs f32to16 takes an f32), and Math.round(x/d) sends halves toward
// +infinity.
static inline double js_round(double x) {
  const double r = std::floor(x);
  return x - r >= 0.5 ? r + 1.0 : r;
}

int flock_quant_q8(const float* w, int64_t rows, int64_t cols, uint8_t* out) {
  if (!w || !out || rows < 1 || cols < 32 || cols % 32) {
    set_error("quantMatrixQ8: cols %lld must be a positive multiple of 32", (long long)cols);
    return FLOCK_E_ARG;
  }
  const int64_t blocks = rows * (cols / 32);
  for (int64_t b = 0; b < blocks; b++) {
    const float* v = w + b * 32;
    uint8_t* o = out + b * 34;
    double amax = 0.0;
    for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs((double)v[i]));
    const double d = amax / 127.0;
    const uint16_t h = f32_to_f16_rne((float)d);
    o[0] = (uint8_t)(h & 0xff);
    o[1] = (uint8_t)(h >> 8);
    for (int i = 0; i < 32; i++) {
      const double q = d == 0.0 ? 0.0 : js_round((double)v[i] / d);
      o[2 + i] = (uint8_t)((int)std::max(-128.0, std::min(127.0, q)) & 0xff);
    }
  }
  return FLOCK_OK;
}

// kernels/lib.ts:64 quantRowQ4 over every row: the scale comes from the first
// value of largest magnitude (strict > scan) so its sign survives.
int flock_quant_q4(const float* w, int64_t rows, int64_t cols, uint8_t* out) {
  if (!w || !out || rows < 1 || cols < 32 || cols % 32) {
    set_error("quantMatrixQ4: cols %lld must be a positive multiple of 32", (long long)cols);
    return FLOCK_E_ARG;
  }
  const int64_t blocks = rows * (cols / 32);
  for (int64_t b = 0; b < blocks; b++) {
    const float* v = w + b * 32;
    uint8_t* o = out + b * 18;
    double amax = 0.0, mx = 0.0;
    for (int i = 0; i < 32; i++) {
      const double a = std::fabs((double)v[i]);
      if (a > amax) {
        amax = a;
        mx = v[i];
      }
    }
    const double d = mx / -8.0;
    const double id = d == 0.0 ? 0.0 : 1.0 / d;
    const uint16_t h = f32_to_f16_rne((float)d);
    o[0] = (uint8_t)(h & 0xff);
    o[1] = (uint8_t)(h >> 8);
    for (int i = 0; i < 16; i++) {
      const double x0 = (double)v[i] * id + 8.5, x1 = (double)v[i + 16] * id + 8.5;
      const int q0 = (int)std::min(15.0, std::max(0.0, std::floor(x0)));
      const int q1 = (int)std::min(15.0, std::max(0.0, std::floor(x1)));
      o[2 + i] = (uint8_t)(q0 | (q1 << 4));
    }
  }
  return FLOCK_OK;
}

}  // extern "C"
