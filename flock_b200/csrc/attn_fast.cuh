// Split-K flash-decode attention for one query token (FLOCK_ATTN_FAST).
//
// Same function as kernels/attention.wgsl:58 / ops_ref.ts:135 attnRef -- GQA
// (query head h reads kv head h / (nH/nKV)), scale 1/sqrt(head_dim),
// max-subtracted softmax over keys 0..pos -- but re-associated for the GPU:
//
//  * grid (kv head g, split s): each CTA owns a contiguous key range of one
//    kv head and serves all G = nH/nKV query heads of that group, so each K/V
//    row is read from HBM once per token, not once per query head;
//  * per split: scores, local max m_s, local sum l_s and unnormalised
//    output o_s (online-softmax partials);
//  * the splits are combined by the last CTA of a group to finish (arrival
//    counter), in both decode engines: out = sum_s o_s e^(m_s-M) /
//    sum_s l_s e^(m_s-M), both sums in split order (af_combine16); each
//    thread combines one output element with all its splits' loads in
//    flight;
//  * a step over n keys uses ceil(n / 32) splits, at most
//    attn_max_splits(SMs, kv heads, cache capacity): 16 for caches of up to
//    2048 keys, caches over 2048 keys run up to 3 CTAs per SM;
//  * scores: one thread per (key, query head), a 128-long dot product over
//    a K tile whose rows are padded to 132 floats (conflict-free 128-bit
//    reads);
//  * before its dependency wait a split stages what no earlier kernel of the
//    step writes (gains, the RoPE row, its first K/V tile), after it only
//    the projection -- one round trip between the wait and the arithmetic.
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
  void* kcache;    // [maxKeys][nKV][hd], f32 or (kv_bf16) bf16
  void* vcache;
  const int* ctl;  // ctl[0] = pos of this token
  float* out;      // [nH][hd]
  float* part;     // [nH][splits][hd + 2]
  uint32_t* count; // [nKV], zero between launches
  int n_heads, n_kv_heads, head_dim, splits;
  float eps;
  int neox;
  int chunk_cap;   // max keys per split (informational; tiles of 64 are staged)
  int combine;     // 1: the last split of a group combines into out; 0: leave partials
  int kv_bf16;     // 1: the cache holds bf16 (widened into the f32 tiles as staged)
  int kv_fp8;      // 1: the cache holds e4m3 (widened into the f32 tiles as staged)
  PrefetchList pf;
  // RoPE (cos, sin) per position and frequency, [rope_rows][hd / 2], the
  // values norm_rope_warp evaluates in f64 (k_rope_table); positions past
  // rope_rows (or no table) evaluate them in place
  const float2* rope_cs;
  int rope_rows;
  int max_keys;  // cache rows; 0: nothing is staged before the dependency wait
};

constexpr int ATTN_FAST_THREADS = 256;
constexpr int ATTN_TILE = 64;  // keys staged in shared memory per pass

// Most splits a decode step may use: one wave of CTAs over the kv heads --
// one CTA per SM, at most 16 splits, for caches of up to ATTN_LONG_KEYS keys
// (short steps are latency-bound: fewer partials combine sooner, and up to
// 16 combine in one round trip -- 18 splits at 257-320 keys measured 10 us
// per token slower than 16); for longer
// caches several CTAs per SM, so that one CTA's K/V loads overlap another's
// arithmetic, and at most ATTN_MAX_SPLITS (a combining lane holds two).
#ifndef FLOCK_ATTN_CTAS_PER_SM
#define FLOCK_ATTN_CTAS_PER_SM 1
#endif
#ifndef FLOCK_ATTN_LONG_CTAS_PER_SM
#define FLOCK_ATTN_LONG_CTAS_PER_SM 3
#endif
constexpr int ATTN_LONG_KEYS = 2048;
constexpr int ATTN_MAX_SPLITS = 64;
static_assert(4 * ATTN_MAX_SPLITS <= 4 * ATTN_TILE, "combine weights live in the score tile");
__host__ __device__ inline int attn_max_splits(int sm_count, int n_kv_heads, int max_keys) {
  const bool long_cache = max_keys > ATTN_LONG_KEYS;
  const int per_sm = long_cache ? FLOCK_ATTN_LONG_CTAS_PER_SM : FLOCK_ATTN_CTAS_PER_SM;
  const int cap = long_cache ? ATTN_MAX_SPLITS : 16;
  int s = n_kv_heads > 0 ? sm_count * per_sm / n_kv_heads : 1;
  return s < 1 ? 1 : (s > cap ? cap : s);
}

// Splits a step over n_keys keys uses: one per ATTN_SPLIT_KEYS keys, at most
// max_splits.  Both decode engines use this rule, so their partials and
// results are identical.  32 keys per split measured 1-5 us per 0.6B token
// faster than 16 (8 slower) with the split's tile staged before the wait.
#ifndef FLOCK_ATTN_SPLIT_KEYS
#define FLOCK_ATTN_SPLIT_KEYS 32
#endif
constexpr int ATTN_SPLIT_KEYS = FLOCK_ATTN_SPLIT_KEYS;
FLOCK_DEV int attn_splits_for(int n_keys, int max_splits) {
  const int s = (n_keys + ATTN_SPLIT_KEYS - 1) / ATTN_SPLIT_KEYS;
  return s < 1 ? 1 : (s > max_splits ? max_splits : s);
}

// Shared-memory layout (floats): raw q [4][128], raw k/v [2][128], gains
// [2][128], inv_freq [64], normalised q [4][128], new k/v [2][128],
// scores/probabilities [4][TILE], running softmax state [4][4], this
// position's RoPE (cos, sin) [64][2], K tile [TILE][AF_KSTRIDE], V tile
// [TILE][128].
constexpr int AF_KSTRIDE = 132;
constexpr int AF_QRAW = 0, AF_KRAW = 512, AF_VRAW = 640, AF_GQ = 768, AF_GK = 896,
              AF_INV = 1024, AF_QV = 1088, AF_KNEW = 1600, AF_VNEW = 1728,
              AF_SC = 1856, AF_ML = AF_SC + 4 * ATTN_TILE, AF_CS = AF_ML + 16,
              AF_KT = AF_CS + 128, AF_VT = AF_KT + ATTN_TILE * AF_KSTRIDE,
              AF_END = AF_VT + ATTN_TILE * 128;

// The key range of split s for the token at position pos.
struct AfRange {
  int n_keys, splits, k0, k1, nk;
};
FLOCK_DEV AfRange af_range(const AttnFastArgs& a, int s, int pos) {
  AfRange r;
  r.n_keys = pos + 1;
  r.splits = attn_splits_for(r.n_keys, a.splits);
  const int chunk = (r.n_keys + r.splits - 1) / r.splits;
  r.k0 = s * chunk;
  r.k1 = min(r.n_keys, r.k0 + chunk);
  r.nk = max(0, r.k1 - r.k0);
  return r;
}

// keys [t0, t0 + nt) of kv head g into the K / V tiles; position pos (this
// token's key, not yet in the cache) is skipped: its row comes from the
// projection.  L2-direct loads: the rows are earlier steps' appends.
// KV: the cache element when known at compile time (0 f32, 1 bf16, 2 e4m3),
// -1: read from the arguments
template <int KV = -1>
FLOCK_DEV void af_stage_tile(const AttnFastArgs& a, int g, int pos, int t0, int nt, float* dsm) {
  const bool fp8 = KV < 0 ? a.kv_fp8 != 0 : KV == 2;
  const bool bf16 = KV < 0 ? a.kv_bf16 != 0 : KV == 1;
  const int t = threadIdx.x;
  const size_t kvs = (size_t)a.n_kv_heads * 128;
  if (fp8) {
    // 8 x 128-bit loads per 128-byte e4m3 row, widened to f32 in the tiles
    for (int i = t; i < nt * 8; i += ATTN_FAST_THREADS) {
      const int j = i >> 3, c16 = i & 7, key = t0 + j;
      if (key == pos) continue;
      const size_t off = (size_t)key * kvs + (size_t)g * 128;
      const uint4 kw = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.kcache) + off) + c16);
      const uint4 vw = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.vcache) + off) + c16);
      fp8x16_widen(kw, dsm + AF_KT + j * AF_KSTRIDE + 16 * c16);
      fp8x16_widen(vw, dsm + AF_VT + j * 128 + 16 * c16);
    }
    return;
  }
  if (bf16) {
    // 16 x 128-bit loads per 256-byte bf16 row, widened to f32 in the tiles
    for (int i = t; i < nt * 16; i += ATTN_FAST_THREADS) {
      const int j = i >> 4, c8 = i & 15, key = t0 + j;
      if (key == pos) continue;
      const size_t off = (size_t)key * kvs + (size_t)g * 128;
      const uint4 kw = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.kcache) + off) + c8);
      const uint4 vw = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.vcache) + off) + c8);
      bf16x8_widen(kw, dsm + AF_KT + j * AF_KSTRIDE + 8 * c8);
      bf16x8_widen(vw, dsm + AF_VT + j * 128 + 8 * c8);
    }
    return;
  }
  for (int i = t; i < nt * 32; i += ATTN_FAST_THREADS) {
    const int j = i >> 5, c4 = i & 31, key = t0 + j;
    if (key == pos) continue;
    const float4* kr = reinterpret_cast<const float4*>(static_cast<const float*>(a.kcache) +
                                                       key * kvs + (size_t)g * 128);
    const float4* vr = reinterpret_cast<const float4*>(static_cast<const float*>(a.vcache) +
                                                       key * kvs + (size_t)g * 128);
    reinterpret_cast<float4*>(dsm + AF_KT)[j * (AF_KSTRIDE / 4) + c4] = __ldcg(kr + c4);
    reinterpret_cast<float4*>(dsm + AF_VT)[i] = __ldcg(vr + c4);
  }
}

// What a split stages that no earlier kernel of the step writes: the q/k
// gains, inverse frequencies, this position's RoPE (cos, sin) row and the
// first K/V tile of the split's keys (rows earlier steps appended).  Safe to
// run before griddepcontrol.wait with a position read there: the step's own
// rows (position pos) are never read from the cache, and the decode graph
// cannot keep the kernel that appended row pos - 1 (the same layer one step
// earlier, ~5 x layers launches back) running while this one starts -- every
// launch between them would have to be resident at once, waiting.
template <int KV = -1>
FLOCK_DEV void af_stage_static(const AttnFastArgs& a, int g, int s, int pos, float* dsm) {
  const int t = threadIdx.x;
  const AfRange r = af_range(a, s, pos);
  const bool fused = a.q_norm != nullptr;
  if (t < 32 && fused) {
    reinterpret_cast<float4*>(dsm + AF_GQ)[t] = reinterpret_cast<const float4*>(a.q_norm)[t];
    reinterpret_cast<float4*>(dsm + AF_GK)[t] = reinterpret_cast<const float4*>(a.k_norm)[t];
    if (t < 16)
      reinterpret_cast<float4*>(dsm + AF_INV)[t] = reinterpret_cast<const float4*>(a.inv_freq)[t];
    if (a.rope_cs != nullptr && pos < a.rope_rows)  // 64 (cos, sin) pairs: 32 float4
      reinterpret_cast<float4*>(dsm + AF_CS)[t] =
          reinterpret_cast<const float4*>(a.rope_cs + (size_t)pos * 64)[t];
  }
  af_stage_tile<KV>(a, g, pos, r.k0, min(r.nk, ATTN_TILE), dsm);
}

// What the step's earlier kernels wrote: the raw q/k/v projection (fused
// norm + RoPE), or the normalised q and the appended k/v row at pos.
template <int KV = -1>
FLOCK_DEV void af_stage_step(const AttnFastArgs& a, int g, int pos, float* dsm) {
  const bool fp8 = KV < 0 ? a.kv_fp8 != 0 : KV == 2;
  const bool bf16 = KV < 0 ? a.kv_bf16 != 0 : KV == 1;
  const int G = a.n_heads / a.n_kv_heads;
  const int t = threadIdx.x;
  const float* qsrc = a.q + (size_t)g * G * 128;
  for (int i = t; i < G * 32; i += ATTN_FAST_THREADS)
    reinterpret_cast<float4*>(dsm + AF_QRAW)[i] = __ldcg(reinterpret_cast<const float4*>(qsrc) + i);
  if (t >= 32) return;
  if (a.q_norm != nullptr) {
    reinterpret_cast<float4*>(dsm + AF_KRAW)[t] =
        __ldcg(reinterpret_cast<const float4*>(a.k + (size_t)g * 128) + t);
    reinterpret_cast<float4*>(dsm + AF_VRAW)[t] =
        __ldcg(reinterpret_cast<const float4*>(a.v + (size_t)g * 128) + t);
    return;
  }
  const size_t off = (size_t)pos * a.n_kv_heads * 128 + (size_t)g * 128;
  if (fp8) {
    if (t < 8) {
      fp8x16_widen(__ldcg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.kcache) + off) + t),
                   dsm + AF_KNEW + 16 * t);
      fp8x16_widen(__ldcg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.vcache) + off) + t),
                   dsm + AF_VNEW + 16 * t);
    }
  } else if (bf16) {
    if (t < 16) {
      bf16x8_widen(__ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.kcache) + off) + t),
                   dsm + AF_KNEW + 8 * t);
      bf16x8_widen(__ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.vcache) + off) + t),
                   dsm + AF_VNEW + 8 * t);
    }
  } else {
    reinterpret_cast<float4*>(dsm + AF_KNEW)[t] =
        __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(a.kcache) + off) + t);
    reinterpret_cast<float4*>(dsm + AF_VNEW)[t] =
        __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(a.vcache) + off) + t);
  }
}

// The combine of one output element from its splits' (o, m, l), loaded by
// `get(split, what)` (what: 0 o, 1 m, 2 l): M = max_s m_s, w_s = e^(m_s - M),
// L = sum_s l_s w_s, O = sum_s o_s w_s in split order, out = O / L, for up
// to 16 splits with every load in flight.
template <typename Get>
FLOCK_DEV float af_combine16(int splits, Get get) {
  float ov[16], mv[16], lv[16];
#pragma unroll
  for (int sp = 0; sp < 16; sp++) {
    const bool has = sp < splits;
    ov[sp] = has ? get(sp, 0) : 0.0f;
    mv[sp] = has ? get(sp, 1) : -INFINITY;
    lv[sp] = has ? get(sp, 2) : 0.0f;
  }
  float M = -INFINITY;
#pragma unroll
  for (int sp = 0; sp < 16; sp++) M = fmaxf(M, mv[sp]);
  float O = 0.0f, L = 0.0f;
#pragma unroll
  for (int sp = 0; sp < 16; sp++) {
    if (sp < splits) {
      const float w = expf(mv[sp] - M);
      L = fmaf(lv[sp], w, L);
      O = fmaf(ov[sp], w, O);
    }
  }
  return O / L;
}

// One (kv head g, split s) work item, run by ATTN_FAST_THREADS threads that
// synchronise with `sync()`; `dsm` holds AF_END floats; `last` is a shared
// flag.  `pos` is the position of the token being decoded.  The caller has
// run af_stage_static and af_stage_step for (g, s, pos) -- the first of them
// possibly before its dependency wait -- without a barrier after them.
template <typename Sync, int KV = -1>
FLOCK_DEV void attn_fast_run(const AttnFastArgs& a, int g, int s, int pos, float* dsm,
                             bool* last_flag, Sync sync) {
  const bool fp8 = KV < 0 ? a.kv_fp8 != 0 : KV == 2;
  const bool bf16 = KV < 0 ? a.kv_bf16 != 0 : KV == 1;
  const int G = a.n_heads / a.n_kv_heads;  // <= 4
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  const int hd = 128;
  const size_t kvs = (size_t)a.n_kv_heads * hd;

  const AfRange r = af_range(a, s, pos);
  const int splits = r.splits, k0 = r.k0, k1 = r.k1;
  if (s >= splits) return;  // uniform over the CTA, before any synchronisation
  const bool fused = a.q_norm != nullptr;
  const bool table = fused && a.rope_cs != nullptr && pos < a.rope_rows;
  float* qv = dsm + AF_QV;
  float* knew = dsm + AF_KNEW;
  float* vnew = dsm + AF_VNEW;
  float* sc = dsm + AF_SC;
  float* ml = dsm + AF_ML;  // per head: m, l, correction
  float* kt = dsm + AF_KT;
  float* vt = dsm + AF_VT;
  float o[2] = {0.0f, 0.0f};  // outputs oi = t, t + 256 (G * 128 <= 512)
  sync();
  if (fused) {
    // exact per-head RMSNorm + RoPE (k_qk_norm_rope_append's arithmetic):
    // warps 0..G-1 the query heads, warp G the new key, warp G+1 copies v;
    // with the table the (cos, sin) pairs are the values norm_rope_warp
    // would evaluate in f64: the same bits without the f64 sin and cos
    const float2* cs = reinterpret_cast<const float2*>(dsm + AF_CS);
    if (warp < G) {
      if (table)
        norm_rope_warp_cs(dsm + AF_QRAW + warp * 128, dsm + AF_GQ, a.eps, cs, a.neox,
                          qv + warp * 128, lane);
      else
        norm_rope_warp(dsm + AF_QRAW + warp * 128, dsm + AF_GQ, a.eps, pos, dsm + AF_INV,
                       a.neox, qv + warp * 128, lane);
    } else if (warp == G) {
      if (table)
        norm_rope_warp_cs(dsm + AF_KRAW, dsm + AF_GK, a.eps, cs, a.neox, knew, lane);
      else
        norm_rope_warp(dsm + AF_KRAW, dsm + AF_GK, a.eps, pos, dsm + AF_INV, a.neox, knew, lane);
    } else if (warp == G + 1) {
      for (int i = lane; i < 128; i += 32) vnew[i] = dsm[AF_VRAW + i];
    }
    sync();
    const size_t off = (size_t)pos * kvs + (size_t)g * hd + t;
    if (fp8) {
      // as with bf16: every split rounds its own copy, split 0 appends it
      if (t < 128) {
        const uint8_t kb = fp8_bits(knew[t]), vb = fp8_bits(vnew[t]);
        knew[t] = fp8_widen(kb);
        vnew[t] = fp8_widen(vb);
        if (s == 0) {
          static_cast<uint8_t*>(a.kcache)[off] = kb;
          static_cast<uint8_t*>(a.vcache)[off] = vb;
        }
      }
      sync();
    } else if (bf16) {
      // every split rounds its own copy of the new key/value, so the scores
      // see the value the cache keeps; split 0 appends it
      if (t < 128) {
        const uint16_t kb = bf16_bits(knew[t]), vb = bf16_bits(vnew[t]);
        knew[t] = __uint_as_float((uint32_t)kb << 16);
        vnew[t] = __uint_as_float((uint32_t)vb << 16);
        if (s == 0) {
          static_cast<uint16_t*>(a.kcache)[off] = kb;
          static_cast<uint16_t*>(a.vcache)[off] = vb;
        }
      }
      sync();
    } else if (s == 0 && t < 128) {
      static_cast<float*>(a.kcache)[off] = knew[t];
      static_cast<float*>(a.vcache)[off] = vnew[t];
    }
  } else {
    for (int i = t; i < G * 128; i += ATTN_FAST_THREADS) qv[i] = dsm[AF_QRAW + i];
    sync();
  }

  const float scale = __double2float_rn(1.0 / sqrt((double)hd));
  if (t < G) {
    ml[4 * t] = -INFINITY;
    ml[4 * t + 1] = 0.0f;
  }
  for (int t0 = k0; t0 < k1; t0 += ATTN_TILE) {
    const int nt = min(ATTN_TILE, k1 - t0);
    if (t0 != k0) {
      sync();
      af_stage_tile<KV>(a, g, pos, t0, nt, dsm);
    }
    // the new key/value live in shared memory, not (yet) in the cache
    if (pos >= t0 && pos < t0 + nt && t < 128) {
      kt[(pos - t0) * AF_KSTRIDE + t] = knew[t];
      vt[(pos - t0) * 128 + t] = vnew[t];
    }
    sync();
    // scores: one thread per (query head, key), four partial sums over the
    // components of the 128-bit reads (a compact loop: what runs after the
    // dependency wait is mostly instruction-fetch and latency bound, and a
    // warp-per-dot-product form measured slower)
    for (int idx = t; idx < G * nt; idx += ATTN_FAST_THREADS) {
      const int hq = idx / nt, j = idx - hq * nt;
      const float4* kr = reinterpret_cast<const float4*>(kt + j * AF_KSTRIDE);
      const float4* qr = reinterpret_cast<const float4*>(qv + hq * 128);
      float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f, p3 = 0.0f;
#pragma unroll 8
      for (int c4 = 0; c4 < 32; c4++) {
        const float4 kk = kr[c4], qq = qr[c4];
        p0 = fmaf(qq.x, kk.x, p0);
        p1 = fmaf(qq.y, kk.y, p1);
        p2 = fmaf(qq.z, kk.z, p2);
        p3 = fmaf(qq.w, kk.w, p3);
      }
      sc[hq * ATTN_TILE + j] = ((p0 + p1) + (p2 + p3)) * scale;
    }
    sync();
    // online softmax per head (warp hq): new max, correction, probabilities
    if (warp < G) {
      const int hq = warp;
      float mt = -INFINITY;
      for (int j = lane; j < nt; j += 32) mt = fmaxf(mt, sc[hq * ATTN_TILE + j]);
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o2));
      const float m_old = ml[4 * hq];
      const float m_new = fmaxf(m_old, mt);
      float lt = 0.0f;
      for (int j = lane; j < nt; j += 32) {
        const float pj = expf(sc[hq * ATTN_TILE + j] - m_new);
        sc[hq * ATTN_TILE + j] = pj;
        lt += pj;
      }
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o2);
      __syncwarp();
      if (lane == 0) {
        const float c = expf(m_old - m_new);
        ml[4 * hq] = m_new;
        ml[4 * hq + 1] = fmaf(ml[4 * hq + 1], c, lt);
        ml[4 * hq + 2] = c;
      }
    }
    sync();
    // unnormalised output: thread owns outputs (hq, i) = t, t + 256
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int oi = t + u * ATTN_FAST_THREADS;
      if (oi < G * hd) {
        const int hq = oi / hd, i = oi % hd;
        float acc = o[u] * ml[4 * hq + 2];
        for (int j = 0; j < nt; j++) acc = fmaf(sc[hq * ATTN_TILE + j], vt[j * 128 + i], acc);
        o[u] = acc;
      }
    }
  }

  // this split's partial: unnormalised o, running max m, sum l
#pragma unroll
  for (int u = 0; u < 2; u++) {
    const int oi = t + u * ATTN_FAST_THREADS;
    if (oi < G * hd) {
      const int hq = oi / hd, i = oi % hd;
      float* pp = a.part + ((size_t)(g * G + hq) * a.splits + s) * (hd + 2);  // stride: max splits
      pp[i] = o[u];
      if (i == 0) {
        pp[hd] = ml[4 * hq];
        pp[hd + 1] = ml[4 * hq + 1];
      }
    }
  }
  if (!a.combine) return;  // combined by the caller after a grid-wide barrier
  // arrival: the CTA barrier orders every thread's partial stores before
  // thread 0's release-acquire increment (release is cumulative); the last
  // arrival's acquire, and the barrier after it, order the other splits'
  // stores before the combine's loads
  sync();
  if (t == 0) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.count + g)
                 : "memory");
    *last_flag = old == (uint32_t)(splits - 1);
  }
  sync();
  if (!*last_flag) return;
  // the combine spread over the whole CTA: every thread owns one (head,
  // element) and issues the loads of its element and of its head's (m, l)
  // for every split together, then combines them (af_combine16) -- the same
  // operations in the same split order for every thread of a head
  for (int oi = t; oi < G * hd; oi += ATTN_FAST_THREADS) {
    const int hq = oi / hd, i = oi - hq * hd;
    const float* pp = a.part + (size_t)(g * G + hq) * a.splits * (hd + 2);
    if (splits <= 16) {
      a.out[(size_t)(g * G + hq) * hd + i] = af_combine16(splits, [&](int sp, int what) {
        const float* q = pp + sp * (hd + 2);
        return __ldcg(what == 0 ? q + i : q + hd + (what - 1));
      });
      continue;
    }
    float M = -INFINITY;
    for (int s0 = 0; s0 < splits; s0 += 32) {
      float mv[32];
#pragma unroll
      for (int sp = 0; sp < 32; sp++)
        mv[sp] = s0 + sp < splits ? __ldcg(pp + (s0 + sp) * (hd + 2) + hd) : -INFINITY;
#pragma unroll
      for (int sp = 0; sp < 32; sp++) M = fmaxf(M, mv[sp]);
    }
    float O = 0.0f, L = 0.0f;
    for (int s0 = 0; s0 < splits; s0 += 16) {
      float ov[16], mv[16], lv[16];
#pragma unroll
      for (int sp = 0; sp < 16; sp++) {
        const bool has = s0 + sp < splits;
        const float* q = pp + (s0 + sp) * (hd + 2);
        ov[sp] = has ? __ldcg(q + i) : 0.0f;
        mv[sp] = has ? __ldcg(q + hd) : -INFINITY;
        lv[sp] = has ? __ldcg(q + hd + 1) : 0.0f;
      }
#pragma unroll
      for (int sp = 0; sp < 16; sp++) {
        if (s0 + sp < splits) {
          const float w = expf(mv[sp] - M);
          L = fmaf(lv[sp], w, L);
          O = fmaf(ov[sp], w, O);
        }
      }
    }
    a.out[(size_t)(g * G + hq) * hd + i] = O / L;
  }
  if (t == 0) a.count[g] = 0;
}

// The whole item for callers that stage in place (the persistent kernel).
template <typename Sync>
FLOCK_DEV void attn_fast_item(const AttnFastArgs& a, int g, int s, int pos, float* dsm,
                              bool* last_flag, Sync sync) {
  if (s >= attn_splits_for(pos + 1, a.splits)) return;
  af_stage_static(a, g, s, pos, dsm);
  af_stage_step(a, g, pos, dsm);
  attn_fast_run(a, g, s, pos, dsm, last_flag, sync);
}

struct BlockSync {
  FLOCK_DEV void operator()() const { __syncthreads(); }
};

// Graph decode.  Before the dependency wait each split stages what
// no earlier kernel of the step writes, for the position the step control
// holds then (the step's position for every layer but the first, whose
// earlier kernel advances it); after the wait it reads the position with the
// projection and restages if the position moved.
// KV: the cache element (0 f32, 1 bf16, 2 e4m3) as a compile-time constant,
// so each instance holds only its own cache paths (what runs after the wait
// is bound by instruction fetch; a smaller hot path misses less).
template <int KV>
static __global__ void __launch_bounds__(ATTN_FAST_THREADS) k_attn_decode_fast(const AttnFastArgs a) {
  extern __shared__ __align__(16) float dsm[];
  __shared__ bool last;
  issue_prefetch(a.pf);
  pdl_launch_dependents();
  const int g = blockIdx.x, s = blockIdx.y;
  const int guess = *(volatile const int*)a.ctl;
  const bool pre = guess >= 0 && guess < a.max_keys && s < attn_splits_for(guess + 1, a.splits);
  if (pre) af_stage_static<KV>(a, g, s, guess, dsm);
  pdl_wait();
  // the raw projection's addresses do not depend on the position: with the
  // fused norm its loads go out together with the position's (one round
  // trip), and are staged as af_stage_step stages them once the position
  // says this split has keys
  const bool fused = a.q_norm != nullptr;
  const int G = a.n_heads / a.n_kv_heads, t = threadIdx.x;
  float4 qr = make_float4(0.f, 0.f, 0.f, 0.f), kr = qr, vr = qr;
  if (fused) {
    if (t < G * 32) qr = __ldcg(reinterpret_cast<const float4*>(a.q + (size_t)g * G * 128) + t);
    if (t < 32) {
      kr = __ldcg(reinterpret_cast<const float4*>(a.k + (size_t)g * 128) + t);
      vr = __ldcg(reinterpret_cast<const float4*>(a.v + (size_t)g * 128) + t);
    }
  }
  const int pos = __ldcg(a.ctl);
  const AfRange r = af_range(a, s, pos);
  if (s < r.splits) {
    if (fused) {
      if (t < G * 32) reinterpret_cast<float4*>(dsm + AF_QRAW)[t] = qr;
      if (t < 32) {
        reinterpret_cast<float4*>(dsm + AF_KRAW)[t] = kr;
        reinterpret_cast<float4*>(dsm + AF_VRAW)[t] = vr;
      }
    } else {
      af_stage_step<KV>(a, g, pos, dsm);
    }
    if (!pre || pos != guess) af_stage_static<KV>(a, g, s, pos, dsm);
  }
  attn_fast_run<BlockSync, KV>(a, g, s, pos, dsm, &last, BlockSync{});
}

inline size_t attn_fast_smem(int /*chunk_cap*/) { return (size_t)AF_END * 4; }

}  // namespace flock
