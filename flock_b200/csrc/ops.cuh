// The non-matmul kernels of the decoder layer, in the reference's f32 order.
//
//   k_qk_norm_rope_append  kernels/rmsnorm.wgsl + rope.wgsl + the KV copies of
//                          layer.ts:620-622, fused: per-head RMSNorm (q_norm /
//                          k_norm, ops_ref.ts:20), RoPE (ops_ref.ts:65) at
//                          position pos0 + token, k and v appended to the cache.
//   k_attn_decode_exact    kernels/attention.wgsl / ops_ref.ts:135 attnRef:
//                          two-pass softmax, serial sums in key order.
//   k_attn_prefill_exact   kernels/attention_prefill.wgsl / head_ref.ts:99:
//                          streaming softmax over 64-key tiles, WG = 128 trees.
//   k_embed                kernels/embed.wgsl / head_ref.ts:34.
//   k_rmsnorm, k_add, k_swiglu, k_argmax  the standalone forms used by the
//                          op-level API (rmsnorm.wgsl, elementwise.wgsl,
//                          argmax.wgsl).
#pragma once
#include <cuda_fp16.h>
#include "common.cuh"

namespace flock {

// Tree over 128 values in shared memory (kernels/lib.ts:312 order); all 128
// threads of the block call it; returns the sum to every thread.
FLOCK_DEV float block128_tree_sum(float v, float* red) {
  const int t = threadIdx.x;
  red[t] = v;
  __syncthreads();
  if (t < 64) red[t] = fadd(red[t], red[t + 64]);
  __syncthreads();
  if (t < 32) {
    float w = fadd(red[t], red[t + 32]);
    w = warp_tree_sum(w);
    if (t == 0) red[128] = w;
  }
  __syncthreads();
  const float r = red[128];
  __syncthreads();
  return r;
}

FLOCK_DEV float fmax_js(float a, float b) { return a > b ? a : b; }

// Tree max over 128 values (head_ref.ts:186 treeReduce(part, Math.max)).
FLOCK_DEV float block128_tree_max(float v, float* red) {
  const int t = threadIdx.x;
  red[t] = v;
  __syncthreads();
  if (t < 64) red[t] = fmax_js(red[t], red[t + 64]);
  __syncthreads();
  if (t < 32) {
    float w = fmax_js(red[t], red[t + 32]);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) w = fmax_js(w, __shfl_down_sync(0xffffffffu, w, s));
    if (t == 0) red[128] = w;
  }
  __syncthreads();
  const float r = red[128];
  __syncthreads();
  return r;
}

struct QkArgs {
  const float* q;   // [n][nH][hd] raw projections
  const float* k;   // [n][nKV][hd]
  const float* v;   // [n][nKV][hd]
  const float* q_norm;
  const float* k_norm;
  const float* inv_freq;  // [hd/2]
  float* qn;        // [n][nH][hd] out
  void* kcache;     // [maxKeys][nKV][hd], f32 (bf16 / e4m3 for k_qk_norm_rope_append<1 / 2>)
  void* vcache;
  const int* ctl;   // ctl[0] = pos0
  int n_tokens, n_heads, n_kv_heads, head_dim;
  float eps;
  int neox;
  PrefetchList pf;
  // tensor-core prefill: the f16 K / V^T tile image of the cache (attn_tc.cuh
  // layout, img_tiles 128-key tiles per kv head) gets each new key too, and
  // the f16 image of the rotated queries ([nH][q_tiles] 128-token tiles, the
  // same layout) each query
  uint8_t* kv_img;
  int img_tiles;
  uint8_t* q_img;
  int q_tiles;
  // RoPE (cos, sin) table [rope_rows][hd / 2] (k_rope_table), or null
  const float2* rope_cs;
  int rope_rows;
};

// Byte offset of element (row, 8-element chunk c16) of a 128 x 128 f16
// operand of the tensor-core attention: two 64-column halves of 128-byte
// rows, 16-byte chunk c of row r at c ^ (r % 8) (attn_tc.cuh atc_off).
FLOCK_DEV uint32_t kvimg_off(int row, int c16) {
  return (uint32_t)(c16 >> 3) * (128u * 128u) + (uint32_t)row * 128u +
         (uint32_t)(((c16 & 7) ^ (row & 7)) << 4);
}

// This key's row of the K tile and column of the V^T tile, from the values
// the cache holds (lane l: elements l, l+32, l+64, l+96), rounded to f16.
FLOCK_DEV void kvimg_put(uint8_t* kv_img, int img_tiles, int kvh, int pos, const float (&kf)[4],
                         const float (&vf)[4], int lane) {
  const int kt = pos >> 7, r = pos & 127;
  uint8_t* kdst = kv_img + ((size_t)kvh * img_tiles + kt) * 2 * (128 * 128 * 2);
  uint8_t* vdst = kdst + 128 * 128 * 2;
#pragma unroll
  for (int q = 0; q < 4; q++) {
    const int e = lane + 32 * q;
    *reinterpret_cast<__half*>(kdst + kvimg_off(r, e >> 3) + (e & 7) * 2) = __float2half_rn(kf[q]);
    *reinterpret_cast<__half*>(vdst + kvimg_off(e, r >> 3) + (r & 7) * 2) = __float2half_rn(vf[q]);
  }
}

// One block of 128 threads per (token, head-vector); head_dim must be 128.
// Exact RMSNorm (WG = 128) + RoPE of one 128-vector by one warp, with no
// block synchronisation: lane l holds elements l, l+32, l+64, l+96 -- the
// grouping the WG = 128 tree folds (partials t and t+64, t+32 and t+96, then
// the shuffle tree) -- so NEOX pairs (i, i+64) are lane-local and NORM pairs
// (2i, 2i+1) are neighbouring lanes.  k_qk_norm_rope_append's arithmetic.
FLOCK_DEV void norm_rope_warp(const float* src, const float* gain, float eps, int pos,
                              const float* inv_freq, int neox, float* dst, int lane) {
  float x[4], y[4];
#pragma unroll
  for (int q = 0; q < 4; q++) x[q] = src[lane + 32 * q];
  float v = fadd(fadd(ffma(x[0], x[0], 0.0f), ffma(x[2], x[2], 0.0f)),
                 fadd(ffma(x[1], x[1], 0.0f), ffma(x[3], x[3], 0.0f)));
  v = warp_tree_sum(v);
  v = __shfl_sync(0xffffffffu, v, 0);
  const float scale = rsqrt_f64r(fadd(fdiv(v, 128.0f), eps));
#pragma unroll
  for (int q = 0; q < 4; q++) y[q] = fmul(fmul(x[q], scale), gain[lane + 32 * q]);
  if (neox) {
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const int i = lane + 32 * q;
      const float theta = fmul((float)pos, inv_freq[i]);
      const float c = __double2float_rn(cos((double)theta));
      const float s = __double2float_rn(sin((double)theta));
      const float av = y[q], bv = y[q + 2];
      dst[i] = ffma(-bv, s, fmul(av, c));
      dst[i + 64] = ffma(bv, c, fmul(av, s));
    }
  } else {
    const bool odd = lane & 1;
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int e = lane + 32 * q;
      const float other = __shfl_xor_sync(0xffffffffu, y[q], 1);
      const float av = odd ? other : y[q], bv = odd ? y[q] : other;
      const float theta = fmul((float)pos, inv_freq[e >> 1]);
      const float c = __double2float_rn(cos((double)theta));
      const float s = __double2float_rn(sin((double)theta));
      dst[e] = odd ? ffma(bv, c, fmul(av, s)) : ffma(-bv, s, fmul(av, c));
    }
  }
}

// norm_rope_warp (k_qk_norm_rope_append's arithmetic, bit for bit) with the
// (cos, sin) of this position read from a staged table row instead of
// evaluated in f64: the same rounded values.
FLOCK_DEV void norm_rope_warp_cs(const float* src, const float* gain, float eps,
                                 const float2* cs, int neox, float* dst, int lane) {
  float x[4], y[4];
#pragma unroll
  for (int q = 0; q < 4; q++) x[q] = src[lane + 32 * q];
  float v = fadd(fadd(ffma(x[0], x[0], 0.0f), ffma(x[2], x[2], 0.0f)),
                 fadd(ffma(x[1], x[1], 0.0f), ffma(x[3], x[3], 0.0f)));
  v = warp_tree_sum(v);
  v = __shfl_sync(0xffffffffu, v, 0);
  const float scale = rsqrt_f64r(fadd(fdiv(v, 128.0f), eps));
#pragma unroll
  for (int q = 0; q < 4; q++) y[q] = fmul(fmul(x[q], scale), gain[lane + 32 * q]);
  if (neox) {
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const int i = lane + 32 * q;
      const float2 t = cs[i];
      const float av = y[q], bv = y[q + 2];
      dst[i] = ffma(-bv, t.y, fmul(av, t.x));
      dst[i + 64] = ffma(bv, t.x, fmul(av, t.y));
    }
  } else {
    const bool odd = lane & 1;
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int e = lane + 32 * q;
      const float other = __shfl_xor_sync(0xffffffffu, y[q], 1);
      const float av = odd ? other : y[q], bv = odd ? y[q] : other;
      const float2 t = cs[e >> 1];
      dst[e] = odd ? ffma(bv, t.x, fmul(av, t.y)) : ffma(-bv, t.y, fmul(av, t.x));
    }
  }
}

// (cos, sin) of fr(pos * inv_freq[i]) for i < 64, as norm_rope_warp rounds them.
FLOCK_DEV float2 rope_cs_at(int pos, float inv_freq_i) {
  const float theta = fmul((float)pos, inv_freq_i);
  return make_float2(__double2float_rn(cos((double)theta)), __double2float_rn(sin((double)theta)));
}

// Builds the RoPE table: rows [0, n_pos) x 64 frequencies.
static __global__ void k_rope_table(const float* inv_freq, int n_pos, float2* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_pos * 64) out[i] = rope_cs_at(i >> 6, inv_freq[i & 63]);
}

// One warp per 128-vector (8 per CTA): q heads -> qn, k heads -> the cache at
// position pos0 + token with v copied beside it.  norm_rope_warp's arithmetic
// is the WG = 128 RMSNorm and RoPE above, bit for bit.  KV: the cache's
// element (FLOCK_KV_F32 / _BF16 / _FP8); for bf16 and e4m3 the rotated key is
// staged in shared memory and stored rounded to nearest even, as is v.
template <int KV>
static __global__ void __launch_bounds__(256) k_qk_norm_rope_append(const QkArgs a) {
  __shared__ __align__(16) float kstage[KV != 0 ? 8 * 128 : 4];
  issue_prefetch(a.pf);
  pdl_launch_dependents();
  pdl_wait();
  const int nvec = a.n_heads + a.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vidx = blockIdx.x * 8 + warp;
  if (vidx >= a.n_tokens * nvec) return;
  const int tok = vidx / nvec, hv = vidx % nvec, hd = a.head_dim;
  const bool is_q = hv < a.n_heads;
  const int kvh = hv - a.n_heads;
  const int pos = a.ctl[0] + tok;
  // the table's (cos, sin) are the values norm_rope_warp evaluates in f64
  const bool table = a.rope_cs != nullptr && pos < a.rope_rows;
  const float2* cs = table ? a.rope_cs + (size_t)pos * 64 : nullptr;
  if (is_q) {
    float* qd = a.qn + ((size_t)tok * a.n_heads + hv) * hd;
    if (table)
      norm_rope_warp_cs(a.q + ((size_t)tok * a.n_heads + hv) * hd, a.q_norm, a.eps, cs, a.neox, qd,
                        lane);
    else
      norm_rope_warp(a.q + ((size_t)tok * a.n_heads + hv) * hd, a.q_norm, a.eps, pos, a.inv_freq,
                     a.neox, qd, lane);
    if (a.q_img) {
      // this query's row of its 128-token tile, f16 (this lane's own elements)
      uint8_t* qt = a.q_img + ((size_t)hv * a.q_tiles + (tok >> 7)) * (128 * 128 * 2);
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const int e = lane + 32 * q;
        *reinterpret_cast<__half*>(qt + kvimg_off(tok & 127, e >> 3) + (e & 7) * 2) =
            __float2half_rn(qd[e]);
      }
    }
  } else {
    const size_t row = ((size_t)pos * a.n_kv_heads + kvh) * hd;
    const float* k = a.k + ((size_t)tok * a.n_kv_heads + kvh) * hd;
    const float* v = a.v + ((size_t)tok * a.n_kv_heads + kvh) * hd;
    float kf[4], vf[4];  // the values the cache now holds (for the f16 image)
    if constexpr (KV == 2) {
      float* ks = kstage + warp * 128;
      if (table)
        norm_rope_warp_cs(k, a.k_norm, a.eps, cs, a.neox, ks, lane);
      else
        norm_rope_warp(k, a.k_norm, a.eps, pos, a.inv_freq, a.neox, ks, lane);
      __syncwarp();
      uint8_t* kc = static_cast<uint8_t*>(a.kcache) + row;
      uint8_t* vc = static_cast<uint8_t*>(a.vcache) + row;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint8_t kb = fp8_bits(ks[lane + 32 * q]), vb = fp8_bits(v[lane + 32 * q]);
        kc[lane + 32 * q] = kb;
        vc[lane + 32 * q] = vb;
        kf[q] = fp8_widen(kb);
        vf[q] = fp8_widen(vb);
      }
    } else if constexpr (KV == 1) {
      float* ks = kstage + warp * 128;
      if (table)
        norm_rope_warp_cs(k, a.k_norm, a.eps, cs, a.neox, ks, lane);
      else
        norm_rope_warp(k, a.k_norm, a.eps, pos, a.inv_freq, a.neox, ks, lane);
      __syncwarp();
      uint16_t* kc = static_cast<uint16_t*>(a.kcache) + row;
      uint16_t* vc = static_cast<uint16_t*>(a.vcache) + row;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint16_t kb = bf16_bits(ks[lane + 32 * q]), vb = bf16_bits(v[lane + 32 * q]);
        kc[lane + 32 * q] = kb;
        vc[lane + 32 * q] = vb;
        kf[q] = __uint_as_float((uint32_t)kb << 16);
        vf[q] = __uint_as_float((uint32_t)vb << 16);
      }
    } else {
      float* kc = static_cast<float*>(a.kcache) + row;
      if (table)
        norm_rope_warp_cs(k, a.k_norm, a.eps, cs, a.neox, kc, lane);
      else
        norm_rope_warp(k, a.k_norm, a.eps, pos, a.inv_freq, a.neox, kc, lane);
      float* vc = static_cast<float*>(a.vcache) + row;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        vf[q] = v[lane + 32 * q];
        vc[lane + 32 * q] = vf[q];
        kf[q] = kc[lane + 32 * q];  // this lane's own elements of the rotated key
      }
    }
    if (a.kv_img) kvimg_put(a.kv_img, a.img_tiles, kvh, pos, kf, vf, lane);
  }
}

struct AttnArgs {
  const float* q;  // [n][nH][hd] normalised + rotated
  const float* kcache;
  const float* vcache;
  float* out;      // [n][nH][hd]
  const int* ctl;  // ctl[0] = pos0 (keys before this batch)
  int n_tokens, n_heads, n_kv_heads, head_dim;
  PrefetchList pf;
};

// ops_ref.ts:135 attnRef for ONE query per head: one CTA per head, 256
// threads.  Scores are serial FMA chains over head_dim (one key per thread),
// the softmax sum is one serial chain in key order (thread 128), and each of
// the 128 output channels is one serial chain over keys (threads 0..127), all
// exactly as the reference orders them.  Dynamic smem: n_keys floats.
static __global__ void __launch_bounds__(256) k_attn_decode_exact(const AttnArgs a) {
  extern __shared__ float sc[];  // [n_keys] scores, then exp values
  __shared__ float qs[128];
  __shared__ float red[260];
  __shared__ float inv_s;
  issue_prefetch(a.pf);
  pdl_launch_dependents();
  pdl_wait();
  const int h = blockIdx.x, t = threadIdx.x, hd = a.head_dim;
  const int kvh = h / (a.n_heads / a.n_kv_heads);
  const int n_keys = a.ctl[0] + 1;
  const float scale = __double2float_rn(1.0 / sqrt((double)hd));
  if (t < hd) qs[t] = a.q[(size_t)h * hd + t];
  __syncthreads();
  for (int key = t; key < n_keys; key += blockDim.x) {
    const float4* kr =
        reinterpret_cast<const float4*>(a.kcache + ((size_t)key * a.n_kv_heads + kvh) * hd);
    float acc = 0.0f;
    for (int i4 = 0; i4 < hd / 4; i4++) {
      const float4 kv = kr[i4];
      acc = ffma(qs[4 * i4 + 0], kv.x, acc);
      acc = ffma(qs[4 * i4 + 1], kv.y, acc);
      acc = ffma(qs[4 * i4 + 2], kv.z, acc);
      acc = ffma(qs[4 * i4 + 3], kv.w, acc);
    }
    sc[key] = fmul(acc, scale);
  }
  __syncthreads();
  // max (exact in any order)
  float m = -INFINITY;
  for (int key = t; key < n_keys; key += blockDim.x) m = fmax_js(m, sc[key]);
  red[t] = m;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (t < s) red[t] = fmax_js(red[t], red[t + s]);
    __syncthreads();
  }
  const float mx = red[0];
  __syncthreads();
  for (int key = t; key < n_keys; key += blockDim.x) sc[key] = exp_f64r(fsub(sc[key], mx));
  __syncthreads();
  if (t == 128) {
    float sum = 0.0f;
    for (int key = 0; key < n_keys; key++) sum = fadd(sum, sc[key]);
    inv_s = __double2float_rn(1.0 / (double)sum);
  }
  float acc = 0.0f;
  if (t < hd) {
    const float* vr = a.vcache + (size_t)kvh * hd + t;
    const size_t vstride = (size_t)a.n_kv_heads * hd;
    for (int key = 0; key < n_keys; key++) acc = ffma(sc[key], vr[key * vstride], acc);
  }
  __syncthreads();
  if (t < hd) a.out[(size_t)h * hd + t] = fmul(acc, inv_s);
}

// head_ref.ts:99 attnPrefillRef / attention_prefill.wgsl: one CTA of 128
// threads per (head, query); TILE = 64 keys; tree reductions over WG = 128.
static __global__ void __launch_bounds__(128) k_attn_prefill_exact(const AttnArgs a) {
  constexpr int TILE = 64, WG = 128;
  __shared__ float tile_s[TILE];
  __shared__ float red[132];
  __shared__ float qs[128];
  issue_prefetch(a.pf);
  pdl_launch_dependents();
  pdl_wait();
  const int h = blockIdx.x, qi = blockIdx.y, t = threadIdx.x, hd = a.head_dim;
  const int kvh = h / (a.n_heads / a.n_kv_heads);
  const float scale = __double2float_rn(1.0 / sqrt((double)hd));
  const int pos0 = a.ctl[0];
  const int n_keys = pos0 + qi + 1;
  const size_t qbase = ((size_t)qi * a.n_heads + h) * hd;
  if (t < hd) qs[t] = a.q[qbase + t];
  __syncthreads();
  float m = -INFINITY, l = 0.0f, acc = 0.0f;
  const size_t kvstride = (size_t)a.n_kv_heads * hd;
  for (int base = 0; base < n_keys; base += TILE) {
    const int n_this = min(TILE, n_keys - base);
    if (t < n_this) {
      const float4* kr = reinterpret_cast<const float4*>(a.kcache + (base + t) * kvstride +
                                                         (size_t)kvh * hd);
      float s = 0.0f;
      for (int i4 = 0; i4 < hd / 4; i4++) {
        const float4 kv = kr[i4];
        s = ffma(qs[4 * i4 + 0], kv.x, s);
        s = ffma(qs[4 * i4 + 1], kv.y, s);
        s = ffma(qs[4 * i4 + 2], kv.z, s);
        s = ffma(qs[4 * i4 + 3], kv.w, s);
      }
      tile_s[t] = fmul(s, scale);
    }
    __syncthreads();
    // tile max: thread t owns j = t (n_this <= TILE < WG)
    const float tmax = block128_tree_max(t < n_this ? tile_s[t] : -INFINITY, red);
    const float m_new = fmax_js(m, tmax);
    const float corr = exp_f64r(fsub(m, m_new));
    float e = 0.0f;
    if (t < n_this) {
      e = exp_f64r(fsub(tile_s[t], m_new));
    }
    __syncthreads();
    if (t < n_this) tile_s[t] = e;
    const float tsum = block128_tree_sum(fadd(0.0f, e), red);  // ts = fr(0 + e)
    if (t < hd) {
      float av = fmul(acc, corr);
      const float* vr = a.vcache + (size_t)base * kvstride + (size_t)kvh * hd + t;
      for (int j = 0; j < n_this; j++) av = ffma(tile_s[j], vr[j * kvstride], av);
      acc = av;
    }
    l = ffma(l, corr, tsum);
    m = m_new;
    __syncthreads();
  }
  if (t < hd) a.out[qbase + t] = fdiv(acc, l);
}

struct EmbedArgs {
  const uint8_t* qs;   // [vocab][hidden] int8
  const uint16_t* sc;  // [vocab][sc_stride]
  const int32_t* ids;
  float* out;          // [n][hidden]
  int n_tokens, hidden, sc_stride;
  int vocab;           // rows of the table; an id outside it embeds as zeros
  PrefetchList pf;
};

// kernels/embed.wgsl:52: gather one Q8_0 row per token and dequantise it.
// The grid may be wider than n_tokens: the extra CTAs only share the L2
// prefetch of the next kernel's weights, which one CTA would issue slowly.
static __global__ void __launch_bounds__(256) k_embed(const EmbedArgs a) {
  issue_prefetch(a.pf);
  pdl_launch_dependents();
  pdl_wait();
  const int tok = blockIdx.x;
  if (tok >= a.n_tokens) return;
  const int64_t row = a.ids[tok];
  const int n4 = a.hidden / 4;
  if (row < 0 || row >= a.vocab) {  // never read outside the table
    for (int g = threadIdx.x; g < n4; g += blockDim.x)
      reinterpret_cast<float4*>(a.out + (size_t)tok * a.hidden)[g] = make_float4(0, 0, 0, 0);
    return;
  }
  for (int g = threadIdx.x; g < n4; g += blockDim.x) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(a.qs + row * a.hidden + 4 * g);
    const float s = scale_f16(a.sc[row * a.sc_stride + g / 8]);
    float q0, q1, q2, q3;
    dec_i8x4(w, q0, q1, q2, q3);
    float4 o = make_float4(fmul(q0, s), fmul(q1, s), fmul(q2, s), fmul(q3, s));
    reinterpret_cast<float4*>(a.out + (size_t)tok * a.hidden)[g] = o;
  }
}

// kernels/rmsnorm.wgsl:41 standalone: one 128-thread block per vector.
static __global__ void __launch_bounds__(128) k_rmsnorm(const float* x, const float* g, float* out, int n,
                                                 int n_vecs, float eps) {
  __shared__ float red[132];
  const int v = blockIdx.x, t = threadIdx.x;
  const float* xv = x + (size_t)v * n;
  float acc = 0.0f;
  for (int i = t; i < n; i += 128) acc = ffma(xv[i], xv[i], acc);
  const float sum = block128_tree_sum(acc, red);
  const float scale = rsqrt_f64r(fadd(fdiv(sum, (float)n), eps));
  for (int i = t; i < n; i += 128) out[(size_t)v * n + i] = fmul(fmul(xv[i], scale), g[i]);
}

// kernels/elementwise.wgsl:31 add / :23 swiglu
static __global__ void k_add(const float* a, const float* b, float* o, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) o[i] = fadd(a[i], b[i]);
}
static __global__ void k_swiglu(const float* g, const float* u, float* o, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float gv = g[i];
    o[i] = fmul(fdiv(gv, fadd(1.0f, exp_f64r(-gv))), u[i]);
  }
}

// kernels/argmax.wgsl pass1+pass2 as one launch: per-CTA (value, index)
// partials, and the last CTA to arrive reduces them.  Same better() rule.
static __global__ void __launch_bounds__(256) k_argmax(const float* x, int64_t n, float* pval,
                                                uint32_t* pidx, uint32_t* count, float* best_val,
                                                int32_t* best_idx, int64_t index_offset) {
  __shared__ float wv[8];
  __shared__ uint32_t wi[8];
  __shared__ bool last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float bv = -FLT_MAX;
  uint32_t bi = 0xFFFFFFFFu;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const uint32_t ix = (uint32_t)(i + index_offset);
    if (v > bv || (v == bv && ix < bi)) {
      bv = v;
      bi = ix;
    }
  }
  auto reduce = [&](float& v, uint32_t& ix) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, v, s);
      const uint32_t oi = __shfl_down_sync(0xffffffffu, ix, s);
      if (ov > v || (ov == v && oi < ix)) {
        v = ov;
        ix = oi;
      }
    }
    if (lane == 0) {
      wv[warp] = v;
      wi[warp] = ix;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x / 32); w++)
        if (wv[w] > wv[0] || (wv[w] == wv[0] && wi[w] < wi[0])) {
          wv[0] = wv[w];
          wi[0] = wi[w];
        }
    }
    __syncthreads();
  };
  reduce(bv, bi);
  if (threadIdx.x == 0) {
    pval[blockIdx.x] = wv[0];
    pidx[blockIdx.x] = wi[0];
    __threadfence();
    last = atomicAdd(count, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  bv = -FLT_MAX;
  bi = 0xFFFFFFFFu;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
    const float v = ((volatile float*)pval)[i];
    const uint32_t ix = ((volatile uint32_t*)pidx)[i];
    if (v > bv || (v == bv && ix < bi)) {
      bv = v;
      bi = ix;
    }
  }
  reduce(bv, bi);
  if (threadIdx.x == 0) {
    *best_val = wv[0];
    *best_idx = (int32_t)wi[0];
    *count = 0;
  }
}

// Advance a step-control block {pos, n_last} without any other work
// (used where no GEMV precedes attention, e.g. an attention-only op call).
static __global__ void k_ctl_advance(int* ctl, int n) {
  ctl[0] += ctl[1];
  ctl[1] = n;
}

}  // namespace flock
