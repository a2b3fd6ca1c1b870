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
//    as f16 into shared memory, O += P V^T accumulated in TMEM, l += sum P;
//    the extra q K^T replaces any rescaling of O;
//  * out = O / l in f32.
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

static __global__ void __launch_bounds__(ATC_THREADS, 1) k_attn_prefill_tc(const AttnTcArgs a) {
  extern __shared__ __align__(16) uint8_t asm_raw[];
  uint8_t* base = asm_raw + ((1024u - (smem_u32(asm_raw) & 1023u)) & 1023u);
  uint8_t* sQ = base;
  uint8_t* sK = sQ + ATC_OPND;
  uint8_t* sV = sK + ATC_OPND;  // V^T: [head_dim][keys]
  uint8_t* sP = sV + ATC_OPND;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sP + ATC_OPND);
  uint64_t* ldbar = bar + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 2);
  __shared__ int s_stop;

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

  if (t == 0) {
    mbar_init(bar, 1);
    mbar_init(ldbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_stop = 0;
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  // q tile (rows past n are zeros)
  atc_stage_row(sQ, t, qi < a.n_tokens ? a.q + ((size_t)qi * a.n_heads + h) * ATC_HD : nullptr);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tS = tmem, tO = tmem + 128;
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
  uint32_t phase = 0, ldphase = 0;
  bool ok = true;

  // K tile kt (and its V^T tile) from the image by bulk copy; everyone waits
  auto stage = [&](int kt, bool with_v) {
    if (t == 0) {
      const uint8_t* src = a.kv_img + ((size_t)g * a.img_tiles + kt) * 2 * ATC_OPND;
      mbar_expect_tx(ldbar, (uint32_t)(with_v ? 2 : 1) * ATC_OPND);
      bulk_g2s(sK, src, ATC_OPND, ldbar);
      if (with_v) bulk_g2s(sV, src + ATC_OPND, ATC_OPND, ldbar);
    }
    if (!mbar_wait(ldbar, ldphase, a.err)) {
      atomicCAS(a.err, 0, 1);
      s_stop = 1;
    }
    ldphase ^= 1;
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

  // ---------------------------------------------------------------- pass 1
  float m = -INFINITY;
  for (int kt = 0; kt < n_tiles && ok; kt++) {
    const int k0 = kt * ATC_K;
    stage(kt, false);
    tc_fence_before();
    __syncthreads();
    scores();
    for (int c0 = 0; c0 < ATC_K; c0 += 16) {
      float s[16];
      tmem_ld16(tS + lane_base + (uint32_t)c0, s);
#pragma unroll
      for (int j = 0; j < 16; j++)
        if (k0 + c0 + j <= qpos) m = fmaxf(m, s[j] * scale);
    }
    tc_fence_before();
    __syncthreads();
    ok = !s_stop;
  }
  // ---------------------------------------------------------------- pass 2
  float l = 0.0f;
  for (int kt = 0; kt < n_tiles && ok; kt++) {
    const int k0 = kt * ATC_K;
    stage(kt, true);
    tc_fence_before();
    __syncthreads();
    scores();
    for (int c0 = 0; c0 < ATC_K; c0 += 16) {
      float s[16];
      tmem_ld16(tS + lane_base + (uint32_t)c0, s);
      float p[16];
#pragma unroll
      for (int j = 0; j < 16; j++) {
        p[j] = k0 + c0 + j <= qpos ? expf(s[j] * scale - m) : 0.0f;
        l += p[j];
      }
#pragma unroll
      for (int half = 0; half < 2; half++)
        *reinterpret_cast<uint4*>(sP + atc_off(t, (c0 >> 3) + half)) =
            make_uint4(h2(p[8 * half], p[8 * half + 1]), h2(p[8 * half + 2], p[8 * half + 3]),
                       h2(p[8 * half + 4], p[8 * half + 5]),
                       h2(p[8 * half + 6], p[8 * half + 7]));
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (t == 0) {
      tc_fence_after();
      atc_mma(tO, smem_u32(sP), smem_u32(sV), kt > 0);
      umma_commit(bar);
    }
    if (!mbar_wait(bar, phase, a.err)) {
      atomicCAS(a.err, 0, 1);
      s_stop = 1;
    }
    phase ^= 1;
    tc_fence_after();
    __syncthreads();
    ok = !s_stop;
  }
  // --------------------------------------------------------------- epilogue
  if (ok) {
    // every lane takes part in the warp-collective loads; rows past n store nothing
    float* dst = a.out + ((size_t)qi * a.n_heads + h) * ATC_HD;
    const float inv = 1.0f / l;
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
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

inline size_t attn_tc_smem_bytes() { return 4 * (size_t)ATC_OPND + 24 + 1024; }

// The f16 image of keys [0, kend) of the cache for k_attn_prefill_tc, kend =
// ctl[0] + n (the position block already advanced for this step): per (key
// tile, kv head) one CTA writes the K tile ([key][head_dim], rows past kend
// zero) and the V^T tile ([head_dim][key]), transposed through shared memory
// so every global load is a coalesced row.  The grid covers the cache's
// capacity; tiles past kend return at once.  BF16: the cache holds bf16,
// widened exactly before the f16 rounding.
constexpr int KVI_STRIDE = 132;  // f32 row stride of the transposition buffer
template <bool BF16>
static __global__ void __launch_bounds__(ATC_THREADS) k_kv_image(const void* kcache,
                                                                const void* vcache,
                                                                int n_kv_heads, const int* ctl,
                                                                int n, int img_tiles,
                                                                uint8_t* img) {
  extern __shared__ __align__(16) float vbuf[];  // [128 keys][KVI_STRIDE]
  const int kt = blockIdx.x, g = blockIdx.y, t = threadIdx.x;
  const int kend = ctl[0] + n;
  if (kt * ATC_K >= kend) return;
  const size_t kvs = (size_t)n_kv_heads * ATC_HD;
  const int key = kt * ATC_K + t;
  const size_t off = (size_t)key * kvs + (size_t)g * ATC_HD;
  uint8_t* kdst = img + ((size_t)g * img_tiles + kt) * 2 * ATC_OPND;
  uint8_t* vdst = kdst + ATC_OPND;
  if constexpr (BF16) {
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
