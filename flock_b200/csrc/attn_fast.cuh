// Split-K flash-decode attention for one query token (FLOCK_ATTN_FAST).
//
// Same function as kernels/attention.wgsl:58 / ops_ref.ts:135 attnRef -- GQA
// (query head h reads kv head h / (nH/nKV)), scale 1/sqrt(head_dim),
// max-subtracted softmax over keys 0..pos -- but re-associated for the GPU:
//
//  * grid (kv head g, split s): each CTA owns a contiguous key range of one
//    kv head and serves all G = nH/nKV query heads of that group, so each K/V
//    row is read from HBM once per token, not once per query head;
//  * per split: scores by warp-parallel dot products, local max m_s, local
//    sum l_s and unnormalised output o_s (online-softmax partials);
//  * the last CTA of a group to finish (arrival counter) combines the splits:
//    out = sum_s o_s e^(m_s-M) / sum_s l_s e^(m_s-M).
//
// There is no key cap (the WGSL decode kernel stops at maxKeys = 2048).  The
// reassociation changes rounding, so parity with attnRef is a tolerance
// (max rel err 1e-5 at the tested sizes), unlike k_attn_decode_exact.
//
// Fused in front: the exact per-head RMSNorm + RoPE of the G query heads and
// of this token's key (k_qk_norm_rope_append's arithmetic, bit for bit), and
// the KV-cache append of the new key/value (by split 0).  The new key is
// also kept in shared memory so splits never race on the cache write.
#pragma once
#include "common.cuh"
#include "ops.cuh"

namespace flock {

struct AttnFastArgs {
  const float* q;  // [nH][hd] raw projection (this token)
  const float* k;  // [nKV][hd]
  const float* v;  // [nKV][hd]
  const float* q_norm;
  const float* k_norm;
  const float* inv_freq;
  float* kcache;
  float* vcache;
  const int* ctl;  // ctl[0] = pos of this token
  float* out;      // [nH][hd]
  float* part;     // [nH][splits][hd + 2]
  uint32_t* count; // [nKV], zero between launches
  int n_heads, n_kv_heads, head_dim, splits;
  float eps;
  int neox;
  int chunk_cap;   // max keys per split this launch was sized for
  PrefetchList pf;
};

// Exact RMSNorm (WG = 128) + RoPE of one 128-vector by one 128-thread half
// of the block; `red` is that half's reduction scratch.  Mirrors
// k_qk_norm_rope_append.  All threads of the block must call it together.
FLOCK_DEV void norm_rope_half(const float* src, const float* gain, float eps, int pos,
                              const float* inv_freq, int neox, float* dst, float* red,
                              float* tmp, bool active) {
  const int t = threadIdx.x & 127;
  const float x = active ? src[t] : 0.0f;
  red[t] = ffma(x, x, 0.0f);
  __syncthreads();
  if (t < 64) red[t] = fadd(red[t], red[t + 64]);
  __syncthreads();
  if (t < 32) {
    float w = fadd(red[t], red[t + 32]);
    w = warp_tree_sum(w);
    if (t == 0) red[128] = w;
  }
  __syncthreads();
  const float scale = rsqrt_f64r(fadd(fdiv(red[128], 128.0f), eps));
  if (active) tmp[t] = fmul(fmul(x, scale), gain[t]);
  __syncthreads();
  if (active && t < 64) {
    const float theta = fmul((float)pos, inv_freq[t]);
    const float c = __double2float_rn(cos((double)theta));
    const float s = __double2float_rn(sin((double)theta));
    const int ia = neox ? t : 2 * t, ib = neox ? t + 64 : 2 * t + 1;
    const float av = tmp[ia], bv = tmp[ib];
    dst[ia] = ffma(-bv, s, fmul(av, c));
    dst[ib] = ffma(bv, c, fmul(av, s));
  }
  __syncthreads();
}

constexpr int ATTN_FAST_THREADS = 256;

static __global__ void __launch_bounds__(ATTN_FAST_THREADS) k_attn_decode_fast(const AttnFastArgs a) {
  extern __shared__ __align__(16) float dsm[];
  const int G = a.n_heads / a.n_kv_heads;  // <= 4
  float* qv = dsm;                          // [G][128]
  float* knew = qv + 4 * 128;               // [128]
  float* vnew = knew + 128;                 // [128]
  float* tmp = vnew + 128;                  // [2][128]
  float* red = tmp + 256;                   // [2][132]
  float* ml = red + 264;                    // [G][2] (m, l)
  float* sc = ml + 8;                       // [G][chunk_cap]
  __shared__ bool last;

  issue_prefetch(a.pf);
  pdl_launch_dependents();
  pdl_wait();

  const int g = blockIdx.x, s = blockIdx.y, t = threadIdx.x;
  const int half = t >> 7, lane = t & 31, warp = t >> 5;
  const int pos = a.ctl[0];
  const int n_keys = pos + 1;
  const int hd = 128;

  if (a.q_norm) {
    // Normalise + rotate the G query heads and the new key (G+1 vectors, two
    // per pass over the two 128-thread halves of the block).
    for (int base = 0; base < G + 1; base += 2) {
      const int vi = base + half;
      const bool active = vi <= G;
      const bool is_k = vi == G;
      const float* src = is_k ? a.k + (size_t)g * hd : a.q + (size_t)(g * G + vi) * hd;
      float* dst = is_k ? knew : qv + vi * 128;
      norm_rope_half(src, is_k ? a.k_norm : a.q_norm, a.eps, pos, a.inv_freq, a.neox, dst,
                     red + half * 132, tmp + half * 128, active);
    }
    if (t < 128) vnew[t] = a.v[(size_t)g * hd + t];
  } else {
    // Pre-normalised form (op-level attention): q is final and the key and
    // value of position pos are already in the cache.
    for (int i = t; i < G * 128; i += ATTN_FAST_THREADS) qv[i] = a.q[(size_t)g * G * hd + i];
    if (t < 128) {
      knew[t] = a.kcache[((size_t)pos * a.n_kv_heads + g) * hd + t];
      vnew[t] = a.vcache[((size_t)pos * a.n_kv_heads + g) * hd + t];
    }
  }
  __syncthreads();
  if (a.q_norm && s == 0 && t < 128) {
    a.kcache[((size_t)pos * a.n_kv_heads + g) * hd + t] = knew[t];
    a.vcache[((size_t)pos * a.n_kv_heads + g) * hd + t] = vnew[t];
  }

  const int chunk = (n_keys + a.splits - 1) / a.splits;
  const int k0 = s * chunk;
  const int k1 = min(n_keys, k0 + chunk);
  const int nk = max(0, k1 - k0);
  const float scale = __double2float_rn(1.0 / sqrt((double)hd));
  const size_t kvs = (size_t)a.n_kv_heads * hd;

  // Scores: one warp per key, float4 per lane, all G heads per K read.
  for (int j = warp; j < nk; j += ATTN_FAST_THREADS / 32) {
    const int key = k0 + j;
    const float4 kv = key == pos ? reinterpret_cast<const float4*>(knew)[lane]
                                 : reinterpret_cast<const float4*>(a.kcache + key * kvs +
                                                                   (size_t)g * hd)[lane];
    for (int hq = 0; hq < G; hq++) {
      const float4 qq = reinterpret_cast<const float4*>(qv + hq * 128)[lane];
      float p = qq.x * kv.x + qq.y * kv.y + qq.z * kv.z + qq.w * kv.w;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
      if (lane == 0) sc[hq * a.chunk_cap + j] = p * scale;
    }
  }
  __syncthreads();
  // Local softmax statistics per head (warp hq).
  if (warp < G) {
    const int hq = warp;
    float m = -INFINITY;
    for (int j = lane; j < nk; j += 32) m = fmaxf(m, sc[hq * a.chunk_cap + j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.0f;
    for (int j = lane; j < nk; j += 32) {
      const float p = expf(sc[hq * a.chunk_cap + j] - m);
      sc[hq * a.chunk_cap + j] = p;
      l += p;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      ml[2 * hq] = m;
      ml[2 * hq + 1] = l;
    }
  }
  __syncthreads();
  // Unnormalised output of this split.
  for (int oi = t; oi < G * hd; oi += ATTN_FAST_THREADS) {
    const int hq = oi / hd, i = oi % hd;
    float acc = 0.0f;
    for (int j = 0; j < nk; j++) {
      const int key = k0 + j;
      const float vv = key == pos ? vnew[i] : a.vcache[key * kvs + (size_t)g * hd + i];
      acc = fmaf(sc[hq * a.chunk_cap + j], vv, acc);
    }
    float* pp = a.part + ((size_t)(g * G + hq) * a.splits + s) * (hd + 2);
    pp[i] = acc;
    if (i == 0) {
      pp[hd] = ml[2 * hq];
      pp[hd + 1] = ml[2 * hq + 1];
    }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) last = atomicAdd(a.count + g, 1u) == (uint32_t)(a.splits - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int oi = t; oi < G * hd; oi += ATTN_FAST_THREADS) {
    const int hq = oi / hd, i = oi % hd;
    const volatile float* pp = a.part + (size_t)(g * G + hq) * a.splits * (hd + 2);
    float M = -INFINITY;
    for (int sp = 0; sp < a.splits; sp++) M = fmaxf(M, pp[sp * (hd + 2) + hd]);
    float L = 0.0f, O = 0.0f;
    for (int sp = 0; sp < a.splits; sp++) {
      const float w = expf(pp[sp * (hd + 2) + hd] - M);
      L = fmaf(pp[sp * (hd + 2) + hd + 1], w, L);
      O = fmaf(pp[sp * (hd + 2) + i], w, O);
    }
    a.out[(size_t)(g * G + hq) * hd + i] = O / L;
  }
  if (t == 0) a.count[g] = 0;
}

inline size_t attn_fast_smem(int chunk_cap) {
  return (size_t)(4 * 128 + 128 + 128 + 256 + 264 + 8 + 4 * chunk_cap) * 4;
}

}  // namespace flock
