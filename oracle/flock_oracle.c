/*
 * flock_oracle.c -- CPU restatement of flock's strict-f32 references.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker, never the product).  Every
 * function names the reference file:line it restates; the header lists them
 * all and explains the arithmetic model.  Compile with -ffp-contract=off.
 */
#include "flock_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_fma_mode = 0;
void fo_set_fma_mode(int mode) { g_fma_mode = mode; }
int fo_get_fma_mode(void) { return g_fma_mode; }

void fo_set_threads(int n) {
#ifdef _OPENMP
  omp_set_num_threads(n < 1 ? 1 : n);
#else
  (void)n;
#endif
}
int fo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Math.fround */
static inline float fr(double x) { return (float)x; }

/* lib.ts:169 fma32: fround(a*b + c) evaluated in f64. */
static inline float fma32(float a, float b, float c) {
  if (g_fma_mode) return fmaf(a, b, c);
  return fr((double)a * (double)b + (double)c);
}

/* lib.ts:196 dot4: one product, then three fma32. */
static inline float dot4(const float* a, const float* b) {
  float s = fr((double)a[0] * (double)b[0]);
  s = fma32(a[1], b[1], s);
  s = fma32(a[2], b[2], s);
  s = fma32(a[3], b[3], s);
  return s;
}

/* lib.ts:312 / ops_ref.ts:176 / shard_ref.ts:252 treeSum: pairwise over a copy. */
static float tree_sum(const float* a, int n) {
  float buf[1024];
  float* b = n <= 1024 ? buf : (float*)malloc(sizeof(float) * (size_t)n);
  memcpy(b, a, sizeof(float) * (size_t)n);
  for (int stride = n >> 1; stride > 0; stride >>= 1)
    for (int i = 0; i < stride; i++) b[i] = fr((double)b[i] + (double)b[i + stride]);
  float r = b[0];
  if (b != buf) free(b);
  return r;
}

/* head_ref.ts:186 treeReduce with Math.max (NaN-propagating like Math.max). */
static double js_max(double a, double b) {
  if (isnan(a) || isnan(b)) return NAN;
  if (a == 0.0 && b == 0.0) return signbit(a) ? b : a; /* max(-0,+0) = +0 */
  return a > b ? a : b;
}
static float tree_max(const float* a, int n) {
  float buf[1024];
  memcpy(buf, a, sizeof(float) * (size_t)n);
  for (int stride = n >> 1; stride > 0; stride >>= 1)
    for (int i = 0; i < stride; i++) buf[i] = (float)js_max(buf[i], buf[i + stride]);
  return buf[0];
}

/* ------------------------------------------------------------------ codecs */

/* lib.ts:30 halfToF32 (inf clamps to the largest finite value). */
double fo_half_to_f32(uint16_t h) {
  double s = (h & 0x8000) ? -1.0 : 1.0;
  int e = (h >> 10) & 0x1f, m = h & 0x3ff;
  if (e == 0) return s * m * ldexp(1.0, -24);
  if (e == 31) return s * 3.4028235e38;
  return s * (1.0 + m / 1024.0) * ldexp(1.0, e - 15);
}

/* wire.mjs:309 f32to16: setFloat32 (round to f32) then RNE to f16 bits. */
uint16_t fo_f32to16(double v) {
  float f = (float)v;
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000;
  int32_t exp = (int32_t)((x >> 23) & 0xff);
  uint32_t man = x & 0x7fffff;
  if (exp == 255) return (uint16_t)(sign | 0x7c00 | (man ? 0x200 : 0));
  exp = exp - 127 + 15;
  if (exp >= 31) return (uint16_t)(sign | 0x7c00);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    man |= 0x800000;
    int shift = 14 - exp;
    uint32_t sub = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
    return (uint16_t)(sign | (sub + ((rem > half || (rem == half && (sub & 1))) ? 1 : 0)));
  }
  uint32_t h = ((uint32_t)exp << 10) | (man >> 13);
  uint32_t rem = man & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h += 1;
  return (uint16_t)(sign | h);
}

/* wire.mjs:333 f16to32 (inf/nan preserved, unlike halfToF32). */
double fo_f16to32(uint16_t h) {
  double s = (h & 0x8000) ? -1.0 : 1.0;
  int e = (h >> 10) & 0x1f, m = h & 0x3ff;
  if (e == 0) return s * m * ldexp(1.0, -24);
  if (e == 31) return m ? NAN : s * INFINITY;
  return s * (1.0 + m / 1024.0) * ldexp(1.0, e - 15);
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline void wr16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xff);
  p[1] = (uint8_t)(v >> 8);
}

/* JS Math.round: nearest integer, halves toward +infinity. */
static double js_round(double x) {
  if (!isfinite(x)) return x;
  double r = floor(x);
  return (x - r >= 0.5) ? r + 1.0 : r;
}

/* --------------------------------------------------------------- quantizers */

/* lib.ts:40 quantRowQ8 */
void fo_quant_row_q8(const float* vals, int64_t n, uint8_t* out) {
  int64_t nb = n / 32;
  for (int64_t b = 0; b < nb; b++) {
    double amax = 0;
    for (int i = 0; i < 32; i++) {
      double a = fabs((double)vals[b * 32 + i]);
      amax = a > amax ? a : amax;
    }
    double d = amax / 127.0;
    wr16(out + b * 34, fo_f32to16(d));
    for (int i = 0; i < 32; i++) {
      double q = d == 0 ? 0 : js_round((double)vals[b * 32 + i] / d);
      if (q < -128) q = -128;
      if (q > 127) q = 127;
      out[b * 34 + 2 + i] = (uint8_t)((int)q & 0xff);
    }
  }
}

/* lib.ts:64 quantRowQ4 */
void fo_quant_row_q4(const float* vals, int64_t n, uint8_t* out) {
  int64_t nb = n / 32;
  for (int64_t b = 0; b < nb; b++) {
    double amax = 0, max = 0;
    for (int i = 0; i < 32; i++) {
      double v = vals[b * 32 + i];
      if (fabs(v) > amax) {
        amax = fabs(v);
        max = v;
      }
    }
    double d = max / -8.0;
    double id = d == 0 ? 0 : 1.0 / d;
    wr16(out + b * 18, fo_f32to16(d));
    for (int i = 0; i < 16; i++) {
      double x0 = (double)vals[b * 32 + i] * id + 8.5;
      double x1 = (double)vals[b * 32 + i + 16] * id + 8.5;
      double f0 = floor(x0), f1 = floor(x1);
      int q0 = (int)fmin(15.0, fmax(0.0, f0));
      int q1 = (int)fmin(15.0, fmax(0.0, f1));
      out[b * 18 + 2 + i] = (uint8_t)(q0 | (q1 << 4));
    }
  }
}

/* lib.ts:94 quantMatrixQ8 */
void fo_quant_matrix_q8(const float* w, int64_t rows, int64_t cols, uint8_t* out) {
  int64_t rb = (cols / 32) * 34;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) fo_quant_row_q8(w + r * cols, cols, out + r * rb);
}

/* lib.ts:103 quantMatrixQ4 */
void fo_quant_matrix_q4(const float* w, int64_t rows, int64_t cols, uint8_t* out) {
  int64_t rb = (cols / 32) * 18;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) fo_quant_row_q4(w + r * cols, cols, out + r * rb);
}

/* lib.ts:126 splitQ8 */
void fo_split_q8(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* qs,
                 uint8_t* scales) {
  int64_t nb = cols / 32, rb = nb * 34;
  for (int64_t r = 0; r < rows; r++)
    for (int64_t b = 0; b < nb; b++) {
      const uint8_t* src = packed + r * rb + b * 34;
      int64_t si = (r * nb + b) * 2;
      scales[si] = src[0];
      scales[si + 1] = src[1];
      memcpy(qs + r * cols + b * 32, src + 2, 32);
    }
}

/* lib.ts:142 splitQ4 */
void fo_split_q4(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* qs,
                 uint8_t* scales) {
  int64_t nb = cols / 32, rb = nb * 18;
  for (int64_t r = 0; r < rows; r++)
    for (int64_t b = 0; b < nb; b++) {
      const uint8_t* src = packed + r * rb + b * 18;
      int64_t si = (r * nb + b) * 2;
      scales[si] = src[0];
      scales[si + 1] = src[1];
      memcpy(qs + (r * nb + b) * 16, src + 2, 16);
    }
}

/* ------------------------------------------------------------------ matvec */

/* One block's decode: lib.ts:265-273 (Q8) and :294-303 (Q4). */
static inline float decode_q8(const uint8_t* base, float* q) {
  for (int i = 0; i < 32; i++) q[i] = (float)(int8_t)base[2 + i];
  return fr(fo_half_to_f32(rd16(base)));
}
static inline float decode_q4(const uint8_t* base, float* q) {
  for (int i = 0; i < 16; i++) {
    uint8_t byte = base[2 + i];
    q[i] = (float)((byte & 0xf) - 8);
    q[i + 16] = (float)((byte >> 4) - 8);
  }
  return fr(fo_half_to_f32(rd16(base)));
}

/* lib.ts:213 matmulF32 for one row: SERIAL (lanes == 0) or coop(lanes).
 * q4 selects the Q4_0 decode and word-pair mapping (lib.ts:307). */
static float matmul_row(const uint8_t* row, const float* x, int64_t cols, int lanes, int q4,
                        float* part) {
  int64_t nb = cols / 32;
  int blk = q4 ? 18 : 34;
  float q[32];
  int L = lanes > 0 ? lanes : 1;
  for (int i = 0; i < L; i++) part[i] = 0.0f;
  for (int64_t b = 0; b < nb; b++) {
    float scale = q4 ? decode_q4(row + b * blk, q) : decode_q8(row + b * blk, q);
    const float* xb = x + b * 32;
    if (lanes == 0) {
      float s = 0.0f;
      for (int i = 0; i < 32; i++) s = fma32(q[i], xb[i], s);
      part[0] = fma32(scale, s, part[0]);
    } else {
      int lane = (int)(b % lanes);
      for (int g = 0; g < 4; g++) {
        /* pair(g): Q8 (g*8..+3, g*8+4..+7); Q4 (g*4..+3, g*4+16..+19) */
        int ia = q4 ? g * 4 : g * 8;
        int ib = q4 ? g * 4 + 16 : g * 8 + 4;
        float d0 = dot4(q + ia, xb + ia);
        float d1 = dot4(q + ib, xb + ib);
        part[lane] = fma32(scale, fr((double)d0 + (double)d1), part[lane]);
      }
    }
  }
  return lanes == 0 ? part[0] : tree_sum(part, lanes);
}

static void matmul_any(const uint8_t* packed, const float* x, int64_t rows, int64_t cols,
                       int lanes, int q4, float* out) {
  int64_t rb = (cols / 32) * (q4 ? 18 : 34);
#pragma omp parallel
  {
    float part[1024];
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; r++) out[r] = matmul_row(packed + r * rb, x, cols, lanes, q4, part);
  }
}

/* lib.ts:251 cpuMatmulQ8F32 */
void fo_matmul_q8(const uint8_t* packed, const float* x, int64_t rows, int64_t cols, int lanes,
                  float* out) {
  matmul_any(packed, x, rows, cols, lanes, 0, out);
}

/* lib.ts:280 cpuMatmulQ4F32 */
void fo_matmul_q4(const uint8_t* packed, const float* x, int64_t rows, int64_t cols, int lanes,
                  float* out) {
  matmul_any(packed, x, rows, cols, lanes, 1, out);
}

/* layer_ref.ts:335 mv(): the per-token matvec N times, concatenated. */
void fo_matmul_q8_batched(const uint8_t* packed, const float* x, int64_t rows, int64_t cols,
                          int n_tokens, int lanes, float* out) {
  for (int t = 0; t < n_tokens; t++)
    matmul_any(packed, x + (int64_t)t * cols, rows, cols, lanes, 0, out + (int64_t)t * rows);
}

/* -------------------------------------------------------------------- ops */

/* ops_ref.ts:20 rmsnormRef */
void fo_rmsnorm(const float* x, const float* g, int n, int n_vecs, double eps, int wg,
                float* out) {
  float part[1024];
  for (int v = 0; v < n_vecs; v++) {
    const float* xv = x + (int64_t)v * n;
    for (int t = 0; t < wg; t++) {
      float acc = 0.0f;
      for (int i = t; i < n; i += wg) acc = fma32(xv[i], xv[i], acc);
      part[t] = acc;
    }
    float sum = tree_sum(part, wg);
    float scale = fr(1.0 / sqrt((double)fr((double)fr((double)sum / (double)n) + eps)));
    for (int i = 0; i < n; i++)
      out[(int64_t)v * n + i] = fr((double)fr((double)xv[i] * (double)scale) * (double)g[i]);
  }
}

/* ops_ref.ts:95 ropeInvFreq (same formula as layer.ts:180 invFreqOf) */
void fo_rope_inv_freq(int head_dim, double base, float* out) {
  int half = head_dim / 2;
  for (int j = 0; j < half; j++) out[j] = fr(1.0 / pow(base, (double)(2 * j) / (double)head_dim));
}

/* ops_ref.ts:65 ropeRef ("neox" pairs halves, "norm" pairs neighbours). */
void fo_rope(const float* x, int n_tokens, int n_heads, int head_dim, int pos0,
             const float* inv_freq, int neox, float* out) {
  int64_t n = (int64_t)n_tokens * n_heads * head_dim;
  memcpy(out, x, sizeof(float) * (size_t)n);
  int half = head_dim / 2;
  for (int t = 0; t < n_tokens; t++)
    for (int h = 0; h < n_heads; h++)
      for (int j = 0; j < half; j++) {
        float theta = fr((double)(pos0 + t) * (double)inv_freq[j]);
        float c = fr(cos((double)theta)), s = fr(sin((double)theta));
        int64_t base = ((int64_t)t * n_heads + h) * head_dim;
        int64_t ia = base + (neox ? j : j * 2);
        int64_t ib = base + (neox ? j + half : j * 2 + 1);
        float a = out[ia], b = out[ib];
        out[ia] = fr(-(double)b * (double)s + (double)fr((double)a * (double)c));
        out[ib] = fr((double)b * (double)c + (double)fr((double)a * (double)s));
      }
}

/* ops_ref.ts:103 swigluRef */
void fo_swiglu(const float* gate, const float* up, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) {
    float g = gate[i];
    float e = fr(exp(-(double)g));
    float den = fr(1.0 + (double)e);
    float sg = fr((double)g / (double)den);
    out[i] = fr((double)sg * (double)up[i]);
  }
}

/* ops_ref.ts:113 addRef */
void fo_add(const float* a, const float* b, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = fr((double)a[i] + (double)b[i]);
}

/* ops_ref.ts:135 attnRef: two-pass softmax, k/v [nKeys][nKV][hd]. */
void fo_attn(const float* q, const float* k, const float* v, int n_heads, int n_kv_heads,
             int head_dim, int n_keys, float* out) {
  int group = n_heads / n_kv_heads;
  float scale = fr(1.0 / sqrt((double)head_dim));
  float* scores = (float*)malloc(sizeof(float) * (size_t)(n_keys > 0 ? n_keys : 1));
  for (int h = 0; h < n_heads; h++) {
    int kvh = h / group;
    for (int t = 0; t < n_keys; t++) {
      float acc = 0.0f;
      const float* kr = k + ((int64_t)t * n_kv_heads + kvh) * head_dim;
      for (int i = 0; i < head_dim; i++) acc = fma32(q[h * head_dim + i], kr[i], acc);
      scores[t] = fr((double)acc * (double)scale);
    }
    double max = -INFINITY;
    for (int t = 0; t < n_keys; t++) max = js_max(max, scores[t]);
    float sum = 0.0f;
    for (int t = 0; t < n_keys; t++) {
      scores[t] = fr(exp((double)fr((double)scores[t] - max)));
      sum = fr((double)sum + (double)scores[t]);
    }
    float inv = fr(1.0 / (double)sum);
    for (int i = 0; i < head_dim; i++) {
      float acc = 0.0f;
      for (int t = 0; t < n_keys; t++)
        acc = fma32(scores[t], v[((int64_t)t * n_kv_heads + kvh) * head_dim + i], acc);
      out[h * head_dim + i] = fr((double)acc * (double)inv);
    }
  }
  free(scores);
}

/* ---------------------------------------------------------------- head ops */

/* head_ref.ts:34 embedRef: gather + dequant from the 34-byte layout. */
void fo_embed(const uint8_t* packed, const int32_t* ids, int n_ids, int cols, float* out) {
  int nb = cols / 32;
  for (int t = 0; t < n_ids; t++) {
    int64_t row = ids[t];
    for (int b = 0; b < nb; b++) {
      const uint8_t* base = packed + (row * nb + b) * 34;
      float scale = fr(fo_half_to_f32(rd16(base)));
      for (int i = 0; i < 32; i++)
        out[(int64_t)t * cols + b * 32 + i] = fr((double)(int8_t)base[2 + i] * (double)scale);
    }
  }
}

/* head_ref.ts:65 argmaxRef: lowest index wins ties. */
int64_t fo_argmax(const float* x, int64_t n) {
  int64_t bi = 0;
  float bv = x[0];
  for (int64_t i = 1; i < n; i++)
    if (x[i] > bv) {
      bv = x[i];
      bi = i;
    }
  return bi;
}

/* head_ref.ts:99 attnPrefillRef: streaming softmax mirroring TILE/WG. */
void fo_attn_prefill(const float* q, const float* k, const float* v, int n_heads, int n_kv_heads,
                     int head_dim, int n_queries, int pos0, int tile, int wg, float* out) {
  int group = n_heads / n_kv_heads;
  float scale = fr(1.0 / sqrt((double)head_dim));
  float* tile_s = (float*)malloc(sizeof(float) * (size_t)tile);
  float* part = (float*)malloc(sizeof(float) * (size_t)wg);
  float* acc = (float*)malloc(sizeof(float) * (size_t)head_dim);
  for (int qi = 0; qi < n_queries; qi++)
    for (int h = 0; h < n_heads; h++) {
      int kvh = h / group;
      int64_t qbase = ((int64_t)qi * n_heads + h) * head_dim;
      int n_keys = pos0 + qi + 1;
      double m = -INFINITY;
      float l = 0.0f;
      for (int i = 0; i < head_dim; i++) acc[i] = 0.0f;
      for (int base = 0; base < n_keys; base += tile) {
        int n_this = tile < n_keys - base ? tile : n_keys - base;
        for (int j = 0; j < n_this; j++) {
          const float* kr = k + ((int64_t)(base + j) * n_kv_heads + kvh) * head_dim;
          float s = 0.0f;
          for (int i = 0; i < head_dim; i++) s = fma32(q[qbase + i], kr[i], s);
          tile_s[j] = fr((double)s * (double)scale);
        }
        for (int t = 0; t < wg; t++) {
          double tm = -INFINITY;
          for (int j = t; j < n_this; j += wg) tm = js_max(tm, tile_s[j]);
          part[t] = (float)tm;
        }
        double tile_max = tree_max(part, wg);
        double m_new = js_max(m, tile_max);
        float corr = fr(exp((double)fr(m - m_new)));
        for (int t = 0; t < wg; t++) {
          float ts = 0.0f;
          for (int j = t; j < n_this; j += wg) {
            float e = fr(exp((double)fr((double)tile_s[j] - m_new)));
            tile_s[j] = e;
            ts = fr((double)ts + (double)e);
          }
          part[t] = ts;
        }
        float tile_sum = tree_sum(part, wg);
        for (int i = 0; i < head_dim; i++) {
          float a = fr((double)acc[i] * (double)corr);
          for (int j = 0; j < n_this; j++)
            a = fma32(tile_s[j], v[((int64_t)(base + j) * n_kv_heads + kvh) * head_dim + i], a);
          acc[i] = a;
        }
        l = fma32(l, corr, tile_sum);
        m = m_new;
      }
      for (int i = 0; i < head_dim; i++) out[qbase + i] = fr((double)acc[i] / (double)l);
    }
  free(tile_s);
  free(part);
  free(acc);
}

/* ------------------------------------------------------------------- layer */

fo_cache* fo_cache_new(int cap, int kvw) {
  fo_cache* c = (fo_cache*)calloc(1, sizeof(fo_cache));
  c->cap = cap;
  c->kvw = kvw;
  c->k = (float*)calloc((size_t)cap * kvw, sizeof(float));
  c->v = (float*)calloc((size_t)cap * kvw, sizeof(float));
  return c;
}
void fo_cache_free(fo_cache* c) {
  if (!c) return;
  free(c->k);
  free(c->v);
  free(c);
}
void fo_cache_reset(fo_cache* c) { c->n = 0; }
int fo_cache_len(const fo_cache* c) { return c->n; }
const float* fo_cache_k(const fo_cache* c) { return c->k; }
const float* fo_cache_v(const fo_cache* c) { return c->v; }
void fo_cache_set_bf16(fo_cache* c, int on) { c->bf16 = on != 0; }
float fo_bf16_round(float x) {
  uint32_t w;
  memcpy(&w, &x, 4);
  if ((w & 0x7fffffffu) > 0x7f800000u) {
    w |= 0x00400000u; /* quiet NaN */
  } else {
    w += 0x7fffu + ((w >> 16) & 1u); /* round to nearest, ties to even */
  }
  w &= 0xffff0000u;
  memcpy(&x, &w, 4);
  return x;
}
void fo_cache_set_fp8(fo_cache* c, int on) { c->bf16 = on ? 2 : 0; }
float fo_fp8_round(float x) {
  if (isnan(x)) return x;
  const float a = fabsf(x);
  if (a >= 448.0f) return copysignf(448.0f, x);
  int e2 = 0;
  frexpf(a, &e2); /* a = f * 2^e2, f in [0.5, 1): a in [2^(e2-1), 2^e2) */
  int E = e2 - 1;
  if (E < -6) E = -6; /* below the smallest normal, 2^-6: subnormal steps of 2^-9 */
  const float step = ldexpf(1.0f, E - 3); /* three mantissa bits */
  /* a / step is exact (a power-of-two scale); rintf rounds ties to even */
  return copysignf(rintf(a / step) * step, x);
}
int fo_cache_fill(fo_cache* c, const float* k, const float* v, int n) {
  if (c->n + n > c->cap) return -1;
  float* kd = c->k + (int64_t)c->n * c->kvw;
  float* vd = c->v + (int64_t)c->n * c->kvw;
  const size_t count = (size_t)n * c->kvw;
  memcpy(kd, k, sizeof(float) * count);
  memcpy(vd, v, sizeof(float) * count);
  if (c->bf16 == 1)
    for (size_t i = 0; i < count; i++) {
      kd[i] = fo_bf16_round(kd[i]);
      vd[i] = fo_bf16_round(vd[i]);
    }
  else if (c->bf16 == 2)
    for (size_t i = 0; i < count; i++) {
      kd[i] = fo_fp8_round(kd[i]);
      vd[i] = fo_fp8_round(vd[i]);
    }
  c->n += n;
  return 0;
}

#define COOP_LANES 64 /* layer_ref.ts:12, must match q8_coop.wgsl */

/* layer_ref.ts:32 layerForwardRef: one decode step, appends to `cache`. */
int fo_layer_forward(const float* hidden, const fo_layer_w* w, const fo_layer_cfg* cfg,
                     fo_cache* cache, float* out) {
  return fo_layer_prefill(hidden, 1, w, cfg, cache, out);
}

/* o_proj / down of one layer: the plain matmul, or (tp > 1) the input-split
 * composition of shard_ref.ts:353 shardedColMatvecRef over tp shards (column
 * ranges of shardRanges(cols, tp, 32), partials summed serially in shard
 * order), token by token. */
static int layer_proj(const uint8_t* packed, const float* x, int64_t rows, int64_t cols, int n,
                      int tp, float* out) {
  if (tp <= 1) {
    fo_matmul_q8_batched(packed, x, rows, cols, n, COOP_LANES, out);
    return 0;
  }
  for (int t = 0; t < n; t++) {
    int rc = fo_sharded_col_matvec(packed, x + (int64_t)t * cols, rows, cols, tp, COOP_LANES,
                                   out + (int64_t)t * rows);
    if (rc) return rc;
  }
  return 0;
}

/* layer_ref.ts:103 layerPrefillRef (n_tokens == 1 is exactly layerForwardRef,
 * whose only difference is attnRef in place of attnPrefillRef). */
int fo_layer_prefill(const float* hidden, int n, const fo_layer_w* w, const fo_layer_cfg* cfg,
                     fo_cache* cache, float* out) {
  return fo_layer_prefill_tp(hidden, n, w, cfg, cache, 1, out);
}

/* layerPrefillRef with o_proj and down replaced by their tp-shard input-split
 * forms (the tensor-parallel layer; tp == 1 is layerPrefillRef itself). */
int fo_layer_prefill_tp(const float* hidden, int n, const fo_layer_w* w, const fo_layer_cfg* cfg,
                        fo_cache* cache, int tp, float* out) {
  const int H = cfg->hidden, nH = cfg->n_heads, nKV = cfg->n_kv_heads, hd = cfg->head_dim,
            F = cfg->ffn;
  const int qw = nH * hd, kvw = nKV * hd;
  if (cache->kvw != kvw) return -1;
  if (cache->n + n > cache->cap) return -1;
  if (tp < 1 || (tp > 1 && ((qw / 32) < tp || (F / 32) < tp))) return -2;
  float inv_freq[512];
  fo_rope_inv_freq(hd, cfg->rope_base, inv_freq);
  int pos0 = cache->n;
  size_t N = (size_t)n;
  float* nh = (float*)malloc(sizeof(float) * N * H);
  float* q = (float*)malloc(sizeof(float) * N * qw);
  float* k = (float*)malloc(sizeof(float) * N * kvw);
  float* v = (float*)malloc(sizeof(float) * N * kvw);
  float* qn = (float*)malloc(sizeof(float) * N * qw);
  float* kn = (float*)malloc(sizeof(float) * N * kvw);
  float* attn = (float*)malloc(sizeof(float) * N * qw);
  float* proj = (float*)malloc(sizeof(float) * N * H);
  float* h2 = (float*)malloc(sizeof(float) * N * H);
  float* gate = (float*)malloc(sizeof(float) * N * F);
  float* up = (float*)malloc(sizeof(float) * N * F);
  float* act = (float*)malloc(sizeof(float) * N * F);

  fo_rmsnorm(hidden, w->attn_norm, H, n, cfg->eps, 128, nh);
  fo_matmul_q8_batched(w->q, nh, qw, H, n, COOP_LANES, q);
  fo_matmul_q8_batched(w->k, nh, kvw, H, n, COOP_LANES, k);
  fo_matmul_q8_batched(w->v, nh, kvw, H, n, COOP_LANES, v);
  fo_rmsnorm(q, w->q_norm, hd, n * nH, cfg->eps, 128, qn);
  fo_rmsnorm(k, w->k_norm, hd, n * nKV, cfg->eps, 128, kn);
  fo_rope(qn, n, nH, hd, pos0, inv_freq, cfg->neox, q);
  fo_rope(kn, n, nKV, hd, pos0, inv_freq, cfg->neox, k);
  fo_cache_fill(cache, k, v, n);
  if (n == 1)
    fo_attn(q, cache->k, cache->v, nH, nKV, hd, cache->n, attn);
  else
    fo_attn_prefill(q, cache->k, cache->v, nH, nKV, hd, n, pos0, 64, 128, attn);
  layer_proj(w->o, attn, H, qw, n, tp, proj);
  fo_add(hidden, proj, N * H, h2);
  fo_rmsnorm(h2, w->ffn_norm, H, n, cfg->eps, 128, nh);
  fo_matmul_q8_batched(w->gate, nh, F, H, n, COOP_LANES, gate);
  fo_matmul_q8_batched(w->up, nh, F, H, n, COOP_LANES, up);
  fo_swiglu(gate, up, N * F, act);
  layer_proj(w->down, act, H, F, n, tp, proj);
  fo_add(h2, proj, N * H, out);

  free(nh); free(q); free(k); free(v); free(qn); free(kn); free(attn);
  free(proj); free(h2); free(gate); free(up); free(act);
  return 0;
}

/* model.ts:307 encodeHead: output_norm once, tied q8 head coop(64), argmax. */
int64_t fo_head(const float* last_row, const float* out_norm, const uint8_t* embd_packed,
                int64_t vocab, int hidden, double eps, float* normed_out, float* logits_out) {
  float* normed = normed_out ? normed_out : (float*)malloc(sizeof(float) * (size_t)hidden);
  float* logits = logits_out ? logits_out : (float*)malloc(sizeof(float) * (size_t)vocab);
  fo_rmsnorm(last_row, out_norm, hidden, 1, eps, 128, normed);
  fo_matmul_q8(embd_packed, normed, vocab, hidden, COOP_LANES, logits);
  int64_t id = fo_argmax(logits, vocab);
  if (!normed_out) free(normed);
  if (!logits_out) free(logits);
  return id;
}

/* ------------------------------------------------------------------- shards */

/* shard_ref.ts:97 shardRanges */
int fo_shard_ranges(int64_t total, int n, int64_t align, int64_t* starts, int64_t* counts) {
  if (n < 1 || total < 0 || align < 1) return -1;
  if (total % align != 0) return -2;
  int64_t units = total / align;
  if (units < n) return -3;
  int64_t base = units / n, extra = units % n, at = 0;
  for (int i = 0; i < n; i++) {
    int64_t count = (base + (i < extra ? 1 : 0)) * align;
    starts[i] = at;
    counts[i] = count;
    at += count;
  }
  return 0;
}

/* shard_ref.ts:137 sliceRows (the reference returns views; this copies them). */
void fo_slice_rows(const uint8_t* qs, const uint8_t* scales, int64_t rows, int64_t cols,
                   int64_t start, int64_t end, uint8_t* qs_out, uint8_t* sc_out) {
  (void)rows;
  int64_t nb = cols / 32;
  memcpy(qs_out, qs + start * cols, (size_t)((end - start) * cols));
  memcpy(sc_out, scales + start * nb * 2, (size_t)((end - start) * nb * 2));
}

/* shard_ref.ts:166 sliceCols */
int fo_slice_cols(const uint8_t* qs, const uint8_t* scales, int64_t rows, int64_t cols,
                  int64_t start, int64_t end, uint8_t* qs_out, uint8_t* sc_out) {
  if (start % 32 || end % 32) return -1;
  if (start < 0 || end > cols || start > end) return -2;
  int64_t nb = cols / 32, w = end - start, wb = w / 32, b0 = start / 32;
  for (int64_t r = 0; r < rows; r++) {
    memcpy(qs_out + r * w, qs + r * cols + start, (size_t)w);
    memcpy(sc_out + r * wb * 2, scales + (r * nb + b0) * 2, (size_t)(wb * 2));
  }
  return 0;
}

/* shard_ref.ts:196 slicePackedCols */
int fo_slice_packed_cols(const uint8_t* packed, int64_t rows, int64_t cols, int64_t start,
                         int64_t end, uint8_t* out) {
  if (start % 32 || end % 32) return -1;
  int64_t nb = cols / 32, wb = (end - start) / 32, b0 = start / 32;
  for (int64_t r = 0; r < rows; r++)
    memcpy(out + r * wb * 34, packed + (r * nb + b0) * 34, (size_t)(wb * 34));
  return 0;
}

/* shard_ref.ts:278 shardMatvecRef: the coop order over the shard's own blocks.
 * Its arithmetic is cpuMatmulQ8F32(coop(lanes)) on the shard's packed bytes. */
void fo_shard_matvec(const uint8_t* packed, const float* x, int64_t rows, int64_t cols, int lanes,
                     float* out) {
  matmul_any(packed, x, rows, cols, lanes, 0, out);
}

/* shard_ref.ts:327 shardReduceRef: serial sum in shard order. parts [n_shards][n]. */
void fo_shard_reduce(const float* parts, int n_shards, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) {
    float acc = parts[i];
    for (int s = 1; s < n_shards; s++) acc = fr((double)acc + (double)parts[(int64_t)s * n + i]);
    out[i] = acc;
  }
}

/* shard_ref.ts:353 shardedColMatvecRef */
int fo_sharded_col_matvec(const uint8_t* packed, const float* x, int64_t rows, int64_t cols,
                          int n_shards, int lanes, float* out) {
  int64_t starts[64], counts[64];
  if (n_shards > 64) return -1;
  int rc = fo_shard_ranges(cols, n_shards, 32, starts, counts);
  if (rc) return rc;
  float* parts = (float*)malloc(sizeof(float) * (size_t)(rows * n_shards));
  for (int s = 0; s < n_shards; s++) {
    uint8_t* sl = (uint8_t*)malloc((size_t)(rows * (counts[s] / 32) * 34));
    fo_slice_packed_cols(packed, rows, cols, starts[s], starts[s] + counts[s], sl);
    fo_shard_matvec(sl, x + starts[s], rows, counts[s], lanes, parts + (int64_t)s * rows);
    free(sl);
  }
  fo_shard_reduce(parts, n_shards, rows, out);
  free(parts);
  return 0;
}

/* shard_ref.ts:378 shardedRowMatvecRef */
int fo_sharded_row_matvec(const uint8_t* packed, const float* x, int64_t rows, int64_t cols,
                          int n_shards, int lanes, float* out) {
  int64_t starts[1024], counts[1024];
  if (n_shards > 1024) return -1;
  int rc = fo_shard_ranges(rows, n_shards, 1, starts, counts);
  if (rc) return rc;
  int64_t rb = (cols / 32) * 34;
  for (int s = 0; s < n_shards; s++)
    fo_shard_matvec(packed + starts[s] * rb, x, counts[s], cols, lanes, out + starts[s]);
  return 0;
}

/* shard_ref.ts:437 reduceShardArgmax */
int64_t fo_reduce_shard_argmax(const float* values, const int64_t* index,
                               const int64_t* row_offset, int n) {
  int64_t bi = -1;
  double bv = -INFINITY;
  for (int p = 0; p < n; p++) {
    int64_t gi = row_offset[p] + index[p];
    if (values[p] > bv || ((double)values[p] == bv && gi < bi)) {
      bv = values[p];
      bi = gi;
    }
  }
  return bi;
}

/* shard_ref.ts:509 memShardPlan */
static double plan_max_binding(int64_t rows, int64_t cols, double bpw, double sbb) {
  double qs = (double)rows * (double)cols * bpw;
  double sc = (double)rows * ceil((double)cols / 32.0) * sbb;
  return qs > sc ? qs : sc;
}
int fo_mem_shard_plan(int64_t rows, int64_t cols, double bpw, double sbb, int n, int dir,
                      double limit, double* max_binding, double* unsharded, int64_t* min_shards,
                      int* fits) {
  int64_t total = dir == 0 ? rows : cols, align = dir == 0 ? 1 : 32;
  int64_t* st = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
  int64_t* ct = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
  int rc = fo_shard_ranges(total, n, align, st, ct);
  if (rc) {
    free(st);
    free(ct);
    return rc;
  }
  double mx = 0;
  for (int i = 0; i < n; i++) {
    double b = dir == 0 ? plan_max_binding(ct[i], cols, bpw, sbb)
                        : plan_max_binding(rows, ct[i], bpw, sbb);
    mx = b > mx ? b : mx;
  }
  free(st);
  free(ct);
  *max_binding = mx;
  *unsharded = plan_max_binding(rows, cols, bpw, sbb);
  *fits = mx <= limit;
  *min_shards = 0;
  int64_t max_n = dir == 0 ? rows : cols / 32;
  for (int64_t kk = 1; kk <= max_n; kk++) {
    /* per-k shard sizes: the max shard is the first one (remainder goes first) */
    int64_t units = total / align;
    int64_t first = (units / kk + (units % kk ? 1 : 0)) * align;
    double m = dir == 0 ? plan_max_binding(first, cols, bpw, sbb)
                        : plan_max_binding(rows, first, bpw, sbb);
    if (m <= limit) {
      *min_shards = kk;
      break;
    }
  }
  return 0;
}

/* ------------------------------------------------------------------ dequant */

/* dequant.ts:22 dequantQ8 */
void fo_dequant_q8(const uint8_t* packed, int64_t rows, int64_t cols, float* out) {
  int64_t nb = cols / 32;
  for (int64_t r = 0; r < rows; r++)
    for (int64_t b = 0; b < nb; b++) {
      const uint8_t* base = packed + (r * nb + b) * 34;
      double scale = fo_half_to_f32(rd16(base));
      for (int i = 0; i < 32; i++)
        out[r * cols + b * 32 + i] = fr((double)(int8_t)base[2 + i] * scale);
    }
}

/* dequant.ts:58 requantWithNoise, one tensor (xorshift32 state carried). */
void fo_requant_with_noise(const uint8_t* packed, int64_t rows, int64_t cols, uint32_t* state,
                           uint8_t* out) {
  float* f = (float*)malloc(sizeof(float) * (size_t)(rows * cols));
  fo_dequant_q8(packed, rows, cols, f);
  int64_t nb = cols / 32;
  uint32_t s = *state;
  for (int64_t r = 0; r < rows; r++)
    for (int64_t b = 0; b < nb; b++) {
      double step = fo_half_to_f32(rd16(packed + (r * nb + b) * 34));
      for (int i = 0; i < 32; i++) {
        s ^= s << 13;
        s ^= s >> 17;
        s ^= s << 5;
        double rnd = ((double)s / 4294967296.0) - 0.5;
        int64_t at = r * cols + b * 32 + i;
        f[at] = fr((double)f[at] + rnd * step);
      }
    }
  *state = s;
  fo_quant_matrix_q8(f, rows, cols, out);
  free(f);
}

/* --------------------------------------------------------------------- wire */

/* wire.mjs:344 pack: "FLK1" | seq | hidden | offset | flags | f16 payload */
int64_t fo_wire_pack(const float* floats, int64_t n, uint32_t seq, uint32_t hidden,
                     uint32_t offset, int reset, int replay, uint8_t* out) {
  uint32_t hdr[5] = {0x314b4c46u, seq, hidden, offset,
                     (uint32_t)((reset ? 1 : 0) | (replay ? 2 : 0))};
  for (int i = 0; i < 5; i++)
    for (int b = 0; b < 4; b++) out[i * 4 + b] = (uint8_t)(hdr[i] >> (8 * b));
  for (int64_t i = 0; i < n; i++) wr16(out + 20 + i * 2, fo_f32to16(floats[i]));
  return 20 + n * 2;
}

/* wire.mjs:358 unpack; meta5 = {seq, hidden, offset, reset, replay}. */
int fo_wire_unpack(const uint8_t* buf, int64_t nbytes, float* out, uint32_t* meta5) {
  uint32_t w[5];
  for (int i = 0; i < 5; i++)
    w[i] = (uint32_t)buf[i * 4] | ((uint32_t)buf[i * 4 + 1] << 8) |
           ((uint32_t)buf[i * 4 + 2] << 16) | ((uint32_t)buf[i * 4 + 3] << 24);
  if (w[0] != 0x314b4c46u) return -1;
  meta5[0] = w[1];
  meta5[1] = w[2];
  meta5[2] = w[3];
  meta5[3] = (w[4] & 1) ? 1 : 0;
  meta5[4] = (w[4] & 2) ? 1 : 0;
  int64_t n = (nbytes - 20) / 2;
  for (int64_t i = 0; i < n; i++) out[i] = (float)fo_f16to32(rd16(buf + 20 + i * 2));
  return 0;
}
