// Causal GQA prefill attention on the tcgen05 tensor cores, for the tensor-
// core prefill path -- kernels/attention_prefill.wgsl:75 / head_ref.ts:99
// attnPrefillRef (queries at positions pos0 .. pos0+n-1, query i sees keys
// 0 .. pos0+i, scale 1/sqrt(head_dim), max-subtracted softmax), re-designed:
//
//  * one CTA per (128-query tile, query head); 4 warps; thread t owns query
//    row t of the tile, which is TMEM lane t of every accumulator, so a row's
//    max and sum need no cross-thread reduction (tcgen05.ld 32x32b);
//  * q is staged as f16 in the K-major 128-byte-swizzled layout (head_dim
//    128 = two 64-wide swizzle chunks); K and V come from an f16 image of the
//    cache that k_kv_image builds once per step (per kv head, 128-key tiles
//    of K and of V transposed to [head_dim][keys], already in that layout),
//    one bulk copy per tile, so both products read K-major operands;
//  * pass 1: S = q K^T per 128-key tile (tcgen05.mma 128x128x16, f32 in
//    TMEM) -> exact row max m;  pass 2: S again, P = e^(S*scale - m) written
//    as f16 into shared memory (over the K tile), O += P V^T accumulated in
//    TMEM, l += sum P; the extra q K^T replaces any rescaling of O.  A range
//    of one key tile needs one S only: its K and V^T copies are issued
//    before the q staging and it runs a single pass;
//  * out = O / l in f32.
//  * the keys of a query tile are cut into gridDim.z contiguous ranges of
//    whole key tiles, one CTA each (the two passes run over the CTA's own
//    range); with more than one range every CTA writes its unnormalised O,
//    its row max m and its sum l, and the o_proj activation image
//    (k_act_image) merges the ranges in order as it reads them (out =
//    sum_z e^(m_z - m) O_z / sum_z e^(m_z - m) l_z), so no extra pass over
//    the output runs.  A 512-token prompt then runs one key tile per CTA
//    over 160 CTAs with work instead of up to four tiles in turn over 64.
//
// Waits are bounded (mbar_wait); on a timeout the kernel sets *err, frees its
// tensor memory and returns.  No multicast is used.
#pragma once
#include "gemm_tc.cuh"

namespace flock {

constexpr int ATC_Q = 128;        // queries per CTA
constexpr int ATC_K = 128;        // keys per tile
constexpr int ATC_HD = 128;       // head_dim (two 64-wide swizzle chunks)
constexpr int ATC_THREADS = 128;
constexpr int ATC_OPND = ATC_Q * ATC_HD * 2;  // bytes of one 128 x 128 f16 operand (32 KiB)

struct AttnTcArgs {
  const float* q;  // [n][nH][hd] normalised + rotated
  const uint8_t* kv_img;  // [nKV][tiles][K tile | V^T tile], ATC_OPND bytes each
  int img_tiles;          // key tiles per kv head in the image
  float* out;      // [n][nH][hd]
  const int* ctl;  // ctl[0] = pos0 (keys before this batch)
  int n_tokens, n_heads, n_kv_heads;
  int* err;
  float* part;     // gridDim.z > 1: [z][n][nH][hd] unnormalised O, then [z][n][nH][2] (m, l)
  // the f16 image of the rotated queries written by the append kernel
  // ([nH][q_tiles] 128-token tiles, the operand layout), or null: q staged
  // from `q` by the threads
  const uint8_t* q_img;
  int q_tiles;
};

// Byte offset of element (row r, column c) -- c < 128 -- in a 128-row operand
// of two 64-column swizzled chunks (16 KiB each).
FLOCK_DEV uint32_t atc_off(int r, int chunk16) {
  return (uint32_t)(chunk16 >> 3) * (ATC_Q * 128) + sw128_off(r, chunk16 & 7);
}

// Row r of a 128 x 128 f16 operand from 128 f32 values at `src` (global),
// or zeros.
FLOCK_DEV void atc_stage_row(uint8_t* op, int r, const float* src) {
#pragma unroll 4
  for (int c = 0; c < 16; c++) {
    uint4 o = make_uint4(0, 0, 0, 0);
    if (src) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src) + 2 * c);
      const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 2 * c + 1);
      o = make_uint4(h2(a.x, a.y), h2(a.z, a.w), h2(b.x, b.y), h2(b.z, b.w));
    }
    *reinterpret_cast<uint4*>(op + atc_off(r, c)) = o;
  }
}

// D (TMEM, 128 lanes x 128 columns) (+)= A . B^T over 128 K elements, both
// 128 x 128 f16 operands in the two-chunk swizzled layout.
FLOCK_DEV void atc_mma(uint32_t d, uint32_t a, uint32_t b, bool accumulate) {
  const uint32_t idesc = umma_idesc_f16(128, 128);
#pragma unroll
  for (int k16 = 0; k16 < 8; k16++) {
    const uint32_t off = (uint32_t)(k16 >> 2) * (ATC_Q * 128) + (uint32_t)(k16 & 3) * 32;
    umma_f16(d, umma_desc_sw128(a + off), umma_desc_sw128(b + off), idesc,
              (accumulate || k16 > 0) ? 1u : 0u);
  }
}

static __global__ void __launch_bounds__(ATC_THREADS, 2) k_attn_prefill_tc(const AttnTcArgs a) {
  extern __shared__ __align__(16) uint8_t asm_raw[];
  uint8_t* base = asm_raw + ((1024u - (smem_u32(asm_raw) & 1023u)) & 1023u);
  uint8_t* sQ = base;
  uint8_t* sK = sQ + ATC_OPND;
  uint8_t* sV = sK + ATC_OPND;  // V^T: [head_dim][keys]
  // P is written over K: S = q K^T has completed (its commit was waited for)
  // before any P store, and the next K lands only after P V^T completed --
  // three operands of shared memory, so two CTAs fit an SM
  uint8_t* sP = sK;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sV + ATC_OPND);
  uint64_t* ldbar = bar + 1;
  uint64_t* qbar = bar + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 3);
  __shared__ int s_stop;
  pdl_wait();

  const int t = threadIdx.x, warp = t >> 5;
  const int h = blockIdx.y, q0 = blockIdx.x * ATC_Q;
  const int G = a.n_heads / a.n_kv_heads, g = h / G;
  const int pos0 = a.ctl[0];
  const int qi = q0 + t;                   // this thread's query
  const int qpos = pos0 + qi;              // its position: sees keys 0..qpos
  const int last_q = min(q0 + ATC_Q, a.n_tokens) - 1;
  const int kend = pos0 + last_q + 1;      // keys any query of the tile sees
  const int n_tiles = (kend + ATC_K - 1) / ATC_K;
  const float scale = __double2float_rn(1.0 / sqrt((double)ATC_HD));
  // this CTA's key tiles [t0, t1)
  const int nz = gridDim.z, z = blockIdx.z;
  const int t0 = z * n_tiles / nz, t1 = (z + 1) * n_tiles / nz;
  const bool single = t1 - t0 == 1;        // one tile: one S, one pass
  float* const part_o = a.part + ((size_t)z * a.n_tokens + qi) * a.n_heads * ATC_HD +
                        (size_t)h * ATC_HD;
  float* const part_ml = a.part + (size_t)nz * a.n_tokens * a.n_heads * ATC_HD +
                         (((size_t)z * a.n_tokens + qi) * a.n_heads + h) * 2;
  if (t0 == t1) {  // no key tile in this range: an empty partial (the merge skips it)
    if (qi < a.n_tokens) {
      part_ml[0] = -INFINITY;
      part_ml[1] = 0.0f;
    }
    return;
  }

  bool inflight = false;  // thread 0: copies issued on ldbar that no wait has seen land
  auto issue = [&](int kt, bool with_v) {  // thread 0: K tile kt (and its V^T) by bulk copy
    inflight = true;
    const uint8_t* src = a.kv_img + ((size_t)g * a.img_tiles + kt) * 2 * ATC_OPND;
    mbar_expect_tx(ldbar, (uint32_t)(with_v ? 2 : 1) * ATC_OPND);
    bulk_g2s(sK, src, ATC_OPND, ldbar);
    if (with_v) bulk_g2s(sV, src + ATC_OPND, ATC_OPND, ldbar);
  };
  const bool qcopy = a.q_img != nullptr;
  bool qinflight = false;  // thread 0: the q copy not yet seen landing
  if (t == 0) {
    mbar_init(bar, 1);
    mbar_init(ldbar, 1);
    mbar_init(qbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_stop = 0;
    if (qcopy) {  // the query tile, one bulk copy
      qinflight = true;
      mbar_expect_tx(qbar, (uint32_t)ATC_OPND);
      bulk_g2s(sQ, a.q_img + ((size_t)h * a.q_tiles + blockIdx.x) * ATC_OPND, ATC_OPND, qbar);
    }
    issue(t0, single);  // the first tile's copies overlap the q staging
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  if (!qcopy) {
    // q tile (rows past n are zeros)
    atc_stage_row(sQ, t, qi < a.n_tokens ? a.q + ((size_t)qi * a.n_heads + h) * ATC_HD : nullptr);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();  // the barriers are initialised, the tensor memory allocated
  tc_fence_after();
  // every CTA holds its tensor memory: a dependent kernel that allocates
  // some may start now without this grid ever waiting on it
  pdl_launch_dependents();
  if (qcopy) {
    // rows past n hold zeros or an earlier step's finite values: their
    // outputs are not stored and rows do not mix in either product
    if (!mbar_wait(qbar, 0, a.err)) {
      atomicCAS(a.err, 0, 1);
      s_stop = 1;
    } else if (t == 0) {
      qinflight = false;
    }
    __syncthreads();  // s_stop agreed on
  }
  const uint32_t tmem = *tslot;
  const uint32_t tS = tmem, tO = tmem + 128;
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
  uint32_t phase = 0, ldphase = 0;
  bool ok = !s_stop;  // the q copy's wait may have given up

  auto land = [&]() {  // everyone: the copies issued on ldbar have landed
    if (!mbar_wait(ldbar, ldphase, a.err)) {
      atomicCAS(a.err, 0, 1);
      s_stop = 1;
    } else {
      inflight = false;
      ldphase ^= 1;
    }
  };
  auto stage = [&](int kt, bool with_v) {
    if (t == 0) issue(kt, with_v);
    land();
  };
  // issue S = q K^T (thread 0) and wait for it (everyone)
  auto scores = [&]() {
    if (t == 0) {
      tc_fence_after();
      atc_mma(tS, smem_u32(sQ), smem_u32(sK), false);
      umma_commit(bar);
    }
    if (!mbar_wait(bar, phase, a.err)) {
      atomicCAS(a.err, 0, 1);
      s_stop = 1;
    }
    phase ^= 1;
    tc_fence_after();
  };
  // the row max of S over this thread's visible keys of tile kt
  auto tile_max = [&](int kt, float m) {
    const int k0 = kt * ATC_K;
    for (int c0 = 0; c0 < ATC_K; c0 += 16) {
      float sv[16];
      tmem_ld16(tS + lane_base + (uint32_t)c0, sv);
#pragma unroll
      for (int j = 0; j < 16; j++)
        if (k0 + c0 + j <= qpos) m = fmaxf(m, sv[j] * scale);
    }
    return m;
  };
  // P = e^(S scale - m) into sP (f16), l += sum P, then O (+)= P V^T
  auto tile_pv = [&](int kt, float m, float& l) {
    const int k0 = kt * ATC_K;
    for (int c0 = 0; c0 < ATC_K; c0 += 16) {
      float sv[16];
      tmem_ld16(tS + lane_base + (uint32_t)c0, sv);
      float p[16];
#pragma unroll
      for (int j = 0; j < 16; j++) {
        p[j] = k0 + c0 + j <= qpos ? expf(sv[j] * scale - m) : 0.0f;
        l += p[j];
      }
#pragma unroll
      for (int hf = 0; hf < 2; hf++)
        *reinterpret_cast<uint4*>(sP + atc_off(t, (c0 >> 3) + hf)) =
            make_uint4(h2(p[8 * hf], p[8 * hf + 1]), h2(p[8 * hf + 2], p[8 * hf + 3]),
                       h2(p[8 * hf + 4], p[8 * hf + 5]), h2(p[8 * hf + 6], p[8 * hf + 7]));
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (t == 0) {
      tc_fence_after();
      atc_mma(tO, smem_u32(sP), smem_u32(sV), kt > t0);
      umma_commit(bar);
    }
    if (!mbar_wait(bar, phase, a.err)) {
      atomicCAS(a.err, 0, 1);
      s_stop = 1;
    }
    phase ^= 1;
    tc_fence_after();
    __syncthreads();
  };

  float m = -INFINITY, l = 0.0f;
  if (single) {
    // K and V^T were issued together: one S, its max, then P and P V^T
    land();
    tc_fence_before();
    __syncthreads();
    ok = !s_stop;
    if (ok) {
      scores();
      m = tile_max(t0, m);
      tile_pv(t0, m, l);
      ok = !s_stop;
    }
  } else {
    // pass 1: the exact row max over the range (K only; the first K was issued)
    for (int kt = t0; kt < t1 && ok; kt++) {
      if (kt == t0) land();
      else stage(kt, false);
      tc_fence_before();
      __syncthreads();
      scores();
      m = tile_max(kt, m);
      tc_fence_before();
      __syncthreads();
      ok = !s_stop;
    }
    // pass 2: S again, P and O += P V^T (no rescaling of O)
    for (int kt = t0; kt < t1 && ok; kt++) {
      stage(kt, true);
      tc_fence_before();
      __syncthreads();
      scores();
      tile_pv(kt, m, l);
      ok = !s_stop;
    }
  }
  // --------------------------------------------------------------- epilogue
  if (ok) {
    // every lane takes part in the warp-collective loads; rows past n store nothing
    const bool whole = nz == 1;
    float* dst = whole ? a.out + ((size_t)qi * a.n_heads + h) * ATC_HD : part_o;
    const float inv = whole ? 1.0f / l : 1.0f;  // a range keeps O unnormalised
    if (!whole && qi < a.n_tokens) {
      part_ml[0] = m;
      part_ml[1] = l;
    }
    for (int c0 = 0; c0 < ATC_HD; c0 += 16) {
      float o[16];
      tmem_ld16(tO + lane_base + (uint32_t)c0, o);
      if (qi < a.n_tokens) {
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(dst + c0 + j) =
              make_float4(o[j] * inv, o[j + 1] * inv, o[j + 2] * inv, o[j + 3] * inv);
      }
    }
  } else if (t == 0) {
    // a wait gave up: let the copies still in flight land before the exit
    if (inflight) mbar_wait(ldbar, ldphase, a.err, false);
    if (qinflight) mbar_wait(qbar, 0, a.err, false);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

inline size_t attn_tc_smem_bytes() { return 3 * (size_t)ATC_OPND + 32 + 1024; }

constexpr int ATC_MAX_SPLITS = 8;  // key ranges per query tile, at most
static_assert(ATC_MAX_SPLITS <= ATC_MAX_SPLITS_IMG, "the o_proj image merges every range");

// Key ranges per query tile for n queries after pos0 cached keys: one key
// tile per CTA as far as ATC_MAX_SPLITS allows (the last query tile sees
// the most tiles).
inline int attn_tc_splits(int pos0_max, int n) {
  const int tiles = (pos0_max + n + ATC_K - 1) / ATC_K;
  return tiles < 1 ? 1 : (tiles > ATC_MAX_SPLITS ? ATC_MAX_SPLITS : tiles);
}


// The f16 image of the cached keys [0, pos0) for k_attn_prefill_tc (pos0 =
// ctl[0]; the step's n new keys are written into the image by
// k_qk_norm_rope_append as it appends them): per (key tile, kv head) one CTA
// writes the K tile ([key][head_dim], rows past kend = pos0 + n zero) and
// the V^T tile ([head_dim][key]), transposed through shared memory so every
// global load is a coalesced row.  The grid covers the tiles holding keys
// before pos0; tiles of new keys only return at once.  KV: the cache's element
// (FLOCK_KV_F32 / _BF16 / _FP8); bf16 and e4m3 are widened exactly before the
// f16 rounding (e4m3 values are f16 values).  Image entries past kend in
// a tile the append wrote hold zeros (the buffer is cleared when allocated)
// or finite values of earlier steps: those keys are masked out of S, and
// their V^T columns meet P = 0.
constexpr int KVI_STRIDE = 132;  // f32 row stride of the transposition buffer
template <int KV>
static __global__ void __launch_bounds__(ATC_THREADS) k_kv_image(const void* kcache,
                                                                const void* vcache,
                                                                int n_kv_heads, const int* ctl,
                                                                int n, int img_tiles,
                                                                uint8_t* img) {
  extern __shared__ __align__(16) float vbuf[];  // [128 keys][KVI_STRIDE]
  pdl_launch_dependents();
  pdl_wait();
  const int kt = blockIdx.x, g = blockIdx.y, t = threadIdx.x;
  const int kend = ctl[0] + n;
  // tiles of new keys only: k_qk_norm_rope_append wrote them (and the tile
  // holding pos0 is rebuilt here whole, its new keys included)
  if (kt * ATC_K >= kend || kt * ATC_K >= ctl[0]) return;
  const size_t kvs = (size_t)n_kv_heads * ATC_HD;
  const int key = kt * ATC_K + t;
  const size_t off = (size_t)key * kvs + (size_t)g * ATC_HD;
  uint8_t* kdst = img + ((size_t)g * img_tiles + kt) * 2 * ATC_OPND;
  uint8_t* vdst = kdst + ATC_OPND;
  if constexpr (KV == 2) {
    const uint4* kr = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(kcache) + off);
    const uint4* vr = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(vcache) + off);
    float kf[16];
#pragma unroll 2
    for (int c = 0; c < 8; c++) {
      uint4 o0 = make_uint4(0, 0, 0, 0), o1 = make_uint4(0, 0, 0, 0);
      if (key < kend) {
        fp8x16_widen(__ldg(kr + c), kf);
        o0 = make_uint4(h2(kf[0], kf[1]), h2(kf[2], kf[3]), h2(kf[4], kf[5]), h2(kf[6], kf[7]));
        o1 = make_uint4(h2(kf[8], kf[9]), h2(kf[10], kf[11]), h2(kf[12], kf[13]), h2(kf[14], kf[15]));
      }
      *reinterpret_cast<uint4*>(kdst + atc_off(t, 2 * c)) = o0;
      *reinterpret_cast<uint4*>(kdst + atc_off(t, 2 * c + 1)) = o1;
    }
#pragma unroll 2
    for (int c = 0; c < 8; c++) {
      float* dst = vbuf + t * KVI_STRIDE + 16 * c;
      if (key < kend) {
        fp8x16_widen(__ldg(vr + c), dst);
      } else {
#pragma unroll
        for (int q = 0; q < 4; q++) reinterpret_cast<float4*>(dst)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  } else if constexpr (KV == 1) {
    const uint4* kr = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(kcache) + off);
    const uint4* vr = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(vcache) + off);
    float kf[8];
#pragma unroll 4
    for (int c = 0; c < 16; c++) {
      uint4 o = make_uint4(0, 0, 0, 0);
      if (key < kend) {
        bf16x8_widen(__ldg(kr + c), kf);
        o = make_uint4(h2(kf[0], kf[1]), h2(kf[2], kf[3]), h2(kf[4], kf[5]), h2(kf[6], kf[7]));
      }
      *reinterpret_cast<uint4*>(kdst + atc_off(t, c)) = o;
    }
#pragma unroll 4
    for (int c = 0; c < 16; c++) {
      float* dst = vbuf + t * KVI_STRIDE + 8 * c;
      if (key < kend) {
        bf16x8_widen(__ldg(vr + c), dst);
      } else {
        reinterpret_cast<float4*>(dst)[0] = make_float4(0.f, 0.f, 0.f, 0.f);
        reinterpret_cast<float4*>(dst)[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  } else {
    const float* kc = static_cast<const float*>(kcache);
    atc_stage_row(kdst, t, key < kend ? kc + off : nullptr);
    const float4* vr = reinterpret_cast<const float4*>(static_cast<const float*>(vcache) + off);
#pragma unroll 8
    for (int c = 0; c < 32; c++)
      reinterpret_cast<float4*>(vbuf + t * KVI_STRIDE)[c] =
          key < kend ? __ldg(vr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  // thread t = head_dim column t of the tile
#pragma unroll 4
  for (int c = 0; c < 16; c++) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = vbuf[(8 * c + e) * KVI_STRIDE + t];
    *reinterpret_cast<uint4*>(vdst + atc_off(t, c)) =
        make_uint4(h2(v[0], v[1]), h2(v[2], v[3]), h2(v[4], v[5]), h2(v[6], v[7]));
  }
}

inline size_t kv_image_smem_bytes() { return (size_t)ATC_K * KVI_STRIDE * 4; }
inline size_t kv_image_bytes(int max_keys, int n_kv_heads) {
  return (size_t)n_kv_heads * ((max_keys + ATC_K - 1) / ATC_K) * 2 * ATC_OPND;
}

}  // namespace flock
