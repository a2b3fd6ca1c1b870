// Streaming persistent decode kernel: one cooperative launch per generated
// token, built for batch-1 latency on B200.
//
// What it computes is the kernel graph's decode step (kernels/model.ts:387
// step -> layer.ts:571 encode per layer -> model.ts:307 encodeHead): the
// embedding gather, per layer RMSNorm + QKV, per-head q/k RMSNorm + RoPE, the
// KV append and GQA attention, o_proj + residual, RMSNorm + gate/up + SwiGLU,
// down + residual, then output_norm, the LM head and its lowest-index argmax.
// Every matvec row is folded in the reference's coop(64) order
// (kernels/lib.ts:213 matmulF32 with coop(64); the same arithmetic as
// k_gemv), so the GEMV outputs are those of the kernel graph bit for bit;
// attention is split-K with an online softmax (a reassociation of
// ops_ref.ts:135 attnRef, held to a tolerance).
//
// How it is laid out:
//
//  * grid = one CTA per SM (cooperative launch, all co-resident), 16 compute
//    warps + 1 producer warp (16 warps: 128 registers a thread);
//  * every CTA owns fixed contiguous row slices of every matrix of every
//    layer and of the head (host-built piece list, `StPiece`).  Weights do
//    not depend on activations, so the producer warp streams the CTA's
//    pieces, in the order they are consumed, into a ring of 16 KiB
//    shared-memory slots with cp.async.bulk (this GPU's memory only, no
//    multicast) and mbarrier completion, as far ahead as the ring allows
//    (about one layer of the 0.6B shape): when a phase's input vector
//    arrives, its rows are already on chip;
//  * activations move between CTAs as tagged 64-bit words (tag << 32 | f32
//    bits) written with one relaxed store each and read with relaxed loads
//    until the tag matches: the word carries its own readiness, so there is
//    no fence, flag or grid barrier between phases -- a consumer waits one L2
//    round trip after the last producer's store.  The tag is (launch
//    sequence << 8 | layer); the dependency chain guarantees a buffer is
//    rewritten only after every reader of its previous value has read it;
//  * attention: items (kv head, split of <= 32-key tiles) on the first CTAs;
//    each normalises and rotates its q heads and the new key (norm_rope_warp,
//    exact), keeps the new key/value on chip and appends it to the cache,
//    stages its K/V tile with loads issued before it waits for q/k/v, and
//    publishes its partial (o, m, l); split 0 combines the group's partials;
//  * the last CTA of the head's argmax writes the id, its history slot, the
//    position and the next launch sequence.
//
// Every wait is bounded (global timer): on a timeout the kernel sets *err,
// stops, lets its bulk copies in flight land, and returns; the host reports
// the error.
#pragma once
#include "common.cuh"
#include "gemv.cuh"
#include "mbar.cuh"
#include "ops.cuh"

namespace flock {

constexpr int ST_CWARPS = 15;
constexpr int ST_CTHREADS = ST_CWARPS * 32;
constexpr int ST_THREADS = ST_CTHREADS + 32;  // + the producer warp
constexpr int ST_SLOT = 16384;                // bytes per ring slot
constexpr int ST_KT = 32;                     // keys per attention tile
constexpr int ST_MAX_SPLITS = 64;
constexpr int ST_PSTRIDE = 132;  // tagged words per (head, split) partial: o[128], m, l, pad
constexpr int ST_MAX_G = 4;      // query heads per kv head

enum { ST_LAST = 1, ST_PAIR = 2 };
enum { ST_ERR_DATA = 4, ST_ERR_RING = 5 };

// One ring slot's worth of one CTA's rows: rows [r, r + nrows) of one matrix
// (and, ST_PAIR, the same rows of a second one: gate | up), laid out in the
// slot as qs_a | sc_a | qs_b | sc_b.  out_row is the first row's index in the
// phase's output vector.  ST_LAST marks the last piece of a phase.
struct StPiece {
  const uint8_t* qs[2];
  const uint16_t* sc[2];
  uint32_t qs_bytes;  // per matrix: nrows * K
  uint32_t sc_bytes;  // per matrix: nrows * sc_stride * 2
  uint32_t out_row;
  uint16_t nrows;
  uint16_t flags;
};
static_assert(sizeof(StPiece) == 48, "StPiece is three 16-byte words");

struct StLayer {
  const float* attn_norm;
  const float* q_norm;
  const float* k_norm;
  const float* ffn_norm;
  void* kcache;  // [max_keys][nKV][hd], f32 or bf16
  void* vcache;
};

struct StArgs {
  const StLayer* layers;
  int n_layers;
  int H, nH, nKV, hd, F, vocab;
  int kv_bf16;
  float eps;
  int neox;
  const float* inv_freq;
  const uint8_t* embd_qs;
  const uint16_t* embd_sc;
  int embd_sc_stride;
  const float* out_norm;
  const StPiece* pieces;  // [grid][max_pieces]
  const int* n_pieces;    // [grid]
  int max_pieces;
  // tagged exchange vectors
  uint64_t* t_qkv;   // [nH*hd + 2*nKV*hd]: q | k | v rows of the QKV projection
  uint64_t* t_part;  // [nH][ST_MAX_SPLITS][ST_PSTRIDE]
  uint64_t* t_att;   // [nH*hd]
  uint64_t* t_ho;    // [H] h after o_proj + residual
  uint64_t* t_act;   // [F]
  uint64_t* t_hd;    // [H] h after down + residual
  float* h_out;      // [H] the last layer's output, plain f32
  float* logits;     // [vocab]
  int32_t* ids;      // ids[0]: the token in, the chosen token out
  int32_t* hist;
  int hist_cap;
  int* ctl;          // {pos of the previous step's first token, n_last}
  unsigned* seq;     // launch sequence number (tags), advanced by the last CTA
  float* am_val;     // [grid]
  uint32_t* am_idx;  // [grid]
  uint32_t* am_count;
  int* err;
  unsigned long long* trace;  // optional: [grid][st_trace_stride(n_layers)] ns
  int splits_max;
  int ring_slots;
  int xbytes;  // bytes of the x-staging / attention union region
};

__host__ __device__ inline int st_trace_stride(int n_layers) { return 4 + 6 * n_layers; }

// ------------------------------------------------------------ primitives
FLOCK_DEV void st_tag(uint64_t* p, uint32_t tag, float v) {
  const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
FLOCK_DEV ulonglong2 st_ld2(const uint64_t* p) {
  ulonglong2 r;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];"
               : "=l"(r.x), "=l"(r.y)
               : "l"(p)
               : "memory");
  return r;
}
FLOCK_DEV uint64_t st_ld1(const uint64_t* p) {
  uint64_t r;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
  return r;
}
FLOCK_DEV uint32_t tag_of(uint64_t w) { return (uint32_t)(w >> 32); }
FLOCK_DEV float val_of(uint64_t w) { return __uint_as_float((uint32_t)w); }

// Named barrier 1 over the compute warps (the producer warp never joins).
FLOCK_DEV void st_bar() { asm volatile("bar.sync 1, %0;" ::"n"(ST_CTHREADS) : "memory"); }
// The same barrier reducing a predicate: true in every compute thread when
// `p` is true in any.  Every fallible step ends with one, so all compute
// threads of a CTA take the same branch and meet the same barriers.
FLOCK_DEV bool st_any(bool p) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)p), "n"(ST_CTHREADS)
      : "memory");
  return r != 0;
}

// Bounded spin for one word pair: true once both tags equal `tag`.
FLOCK_DEV bool st_wait2(const uint64_t* p, uint32_t tag, ulonglong2& w, const int* err) {
  uint64_t t0 = 0;
  for (uint32_t i = 0; tag_of(w.x) != tag || tag_of(w.y) != tag; i++) {
    if ((i & 15) == 15) {
      if (*(volatile const int*)err) return false;
      const uint64_t now = globaltimer_ns();
      if (!t0) t0 = now;
      else if (now - t0 > WAIT_NS) return false;
    }
    __nanosleep(20);
    w = st_ld2(p);
  }
  return true;
}
FLOCK_DEV bool st_wait1(const uint64_t* p, uint32_t tag, uint64_t& w, const int* err) {
  uint64_t t0 = 0;
  for (uint32_t i = 0; tag_of(w) != tag; i++) {
    if ((i & 15) == 15) {
      if (*(volatile const int*)err) return false;
      const uint64_t now = globaltimer_ns();
      if (!t0) t0 = now;
      else if (now - t0 > WAIT_NS) return false;
    }
    __nanosleep(20);
    w = st_ld1(p);
  }
  return true;
}

// The n tagged words at src into dst (PACKED: the Q8_0 packed-pair x layout
// of the folds; else plain), waiting for tag.  All of a thread's loads are
// issued before any is checked.  Called by the compute threads; false (and
// *err set) on a timeout.
template <bool PACKED>
__device__ __noinline__ bool st_poll_vec(const uint64_t* src, int n, uint32_t tag, float* dst, int* err) {
  const int t = threadIdx.x;
  bool ok = true;
  for (int base = 0; base < n / 2; base += 4 * ST_CTHREADS) {
    ulonglong2 w[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int i = base + t + u * ST_CTHREADS;
      if (i < n / 2) w[u] = st_ld2(src + 2 * i);
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int i = base + t + u * ST_CTHREADS;
      if (i >= n / 2) continue;
      if (ok && !st_wait2(src + 2 * i, tag, w[u], err)) {
        ok = false;
        atomicExch(err, ST_ERR_DATA);
      }
      const int e = 2 * i;
      dst[PACKED ? xperm<QT_Q8>(e) : e] = val_of(w[u].x);
      dst[PACKED ? xperm<QT_Q8>(e + 1) : e + 1] = val_of(w[u].y);
    }
  }
  return ok;
}

// ops_ref.ts:20 rmsnormRef with WG = 128 (rmsnorm_to_smem's arithmetic):
// src plain [n] in shared memory, gain staged in gs, result in xs in the
// packed-pair layout.  Called by the compute threads after a barrier that
// made src and gs visible; ends with a barrier.
__device__ __noinline__ void st_rmsnorm(const float* src, const float* gs, int n, float eps, float* xs,
                          float* red) {
  const int t = threadIdx.x;
  if (t < 128) {
    float acc = 0.0f;
    for (int i = t; i < n; i += 128) acc = ffma(src[i], src[i], acc);
    red[t] = acc;
  }
  st_bar();
  if (t < 64) red[t] = fadd(red[t], red[t + 64]);
  st_bar();
  if (t < 32) {
    float v = fadd(red[t], red[t + 32]);
    v = warp_tree_sum(v);
    if (t == 0) red[128] = rsqrt_f64r(fadd(fdiv(v, (float)n), eps));
  }
  st_bar();
  const float scale = red[128];
  for (int i = t; i < n; i += ST_CTHREADS) xs[xperm<QT_Q8>(i)] = fmul(fmul(src[i], scale), gs[i]);
  st_bar();
}

// One Q8_0 row folded from shared memory in gemv_run's lane / block order
// (lane t: blocks t + 32m, m even -> logical lane t, m odd -> lane t + 32;
// then the 64-lane tree): bit-identical to k_gemv.  XREG: the row is one
// block per lane (K <= 1024) and the lane's x pairs are in xp.
template <bool XREG>
FLOCK_DEV float st_row(const uint8_t* q, const uint16_t* s, int nb, const float* xs,
                       const uint64_t (&xp)[16], int lane) {
  float accA = 0.0f, accB = 0.0f;
  if (XREG) {
    if (lane < nb) {
      BlockW<QT_Q8> bw;
      bw.w0 = *reinterpret_cast<const uint4*>(q + lane * 32);
      bw.w1 = *reinterpret_cast<const uint4*>(q + lane * 32 + 16);
      bw.s = s[lane];
      accA = fold_block_packed<QT_Q8>(bw, xp, accA);
    }
  } else {
    const int M = (nb + 31) / 32;
#pragma unroll 1
    for (int m = 0; m < M; m++) {
      const int b = lane + 32 * m;
      if (b >= nb) break;
      BlockW<QT_Q8> bw;
      bw.w0 = *reinterpret_cast<const uint4*>(q + b * 32);
      bw.w1 = *reinterpret_cast<const uint4*>(q + b * 32 + 16);
      bw.s = s[b];
      uint64_t xq[16];
      load_pairs(xs, b, xq);
      if (m & 1)
        accB = fold_block_packed<QT_Q8>(bw, xq, accB);
      else
        accA = fold_block_packed<QT_Q8>(bw, xq, accA);
    }
  }
  return warp_tree_sum(fadd(accA, accB));
}

// Loads the x pairs of this lane's block (K <= 1024 rows) from xs.
FLOCK_DEV void st_xregs(const float* xs, int nb, uint64_t (&xp)[16]) {
  const int lane = threadIdx.x & 31;
  if (lane < nb) {
    load_pairs(xs, lane, xp);
  } else {
#pragma unroll
    for (int j = 0; j < 16; j++) xp[j] = 0;
  }
}

// Shared state of one CTA.
struct StCta {
  uint8_t* ring;
  StPiece* hdr;
  uint64_t* full;
  uint64_t* empty;
  float* xs;   // x staging (packed) | attention tiles
  float* hs;   // [H] plain: the residual stream as this CTA last read it
  float* gs;   // [max(H, F)] gains staging
  float* red;  // [136]
  float* am_v; // [ST_CWARPS]
  uint32_t* am_i;
  int* flags;  // [0]: issued pieces (producer), [1]: last-CTA flag
  int pi;      // consumer's next piece (the same in every compute thread)
};

enum { ST_QKV = 0, ST_O = 1, ST_GU = 2, ST_DOWN = 3, ST_HEAD = 4 };

// The rows of one phase: every piece up to and including the ST_LAST one.
// EPI by phase: QKV -> tagged q|k|v; O / DOWN -> tagged h = hs[row] + y
// (DOWN of the last layer also writes h_out); GU -> tagged SwiGLU(gate, up);
// HEAD -> logits and this warp's argmax (best_v / best_i in lane 0).
// Each phase is compiled on its own (noinline): the row loop gets the
// kernel's whole register budget instead of sharing it with the layer loop.
template <int PH, bool XREG>
__device__ __noinline__ bool st_phase(const StArgs& a, StCta& c, uint32_t tag, bool last_layer,
                                      float* best_out, uint32_t* besti_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t xp[16];
  if (XREG) st_xregs(c.xs, a.H / 32, xp);
  float best_v = -FLT_MAX;
  uint32_t best_i = 0xFFFFFFFFu;
  while (true) {
    const int slot = c.pi % a.ring_slots;
    const uint32_t par = (uint32_t)(c.pi / a.ring_slots) & 1u;
    if (!mbar_wait(&c.full[slot], par, a.err)) {
      if (lane == 0) atomicExch(a.err, ST_ERR_RING);
      return false;
    }
    const StPiece& p = c.hdr[slot];
    const int n = p.nrows;
    const uint16_t flags = p.flags;
    const uint32_t out0 = p.out_row;
    if (n > 0) {
      const int K = (int)(p.qs_bytes / (uint32_t)n);
      const int scs = (int)(p.sc_bytes / (uint32_t)n) / 2;  // halfs per scale row
      const int nb = K / 32;
      const uint8_t* qa = c.ring + (size_t)slot * ST_SLOT;
      const uint16_t* sa = reinterpret_cast<const uint16_t*>(qa + p.qs_bytes);
      const uint8_t* qb = qa + p.qs_bytes + p.sc_bytes;
      const uint16_t* sb = reinterpret_cast<const uint16_t*>(qb + p.qs_bytes);
      for (int r = warp; r < n; r += ST_CWARPS) {
        const float y = st_row<XREG>(qa + (size_t)r * K, sa + (size_t)r * scs, nb, c.xs, xp, lane);
        const uint32_t row = out0 + r;
        if (PH == ST_GU) {
          const float u = st_row<XREG>(qb + (size_t)r * K, sb + (size_t)r * scs, nb, c.xs, xp, lane);
          if (lane == 0) {
            // ops_ref.ts:103 swigluRef: fr(fr(g / fr(1 + fr(exp(-g)))) * up)
            const float e = exp_f64r(-y);
            st_tag(a.t_act + row, tag, fmul(fdiv(y, fadd(1.0f, e)), u));
          }
        } else if (lane == 0) {
          if (PH == ST_QKV) {
            st_tag(a.t_qkv + row, tag, y);
          } else if (PH == ST_O) {
            st_tag(a.t_ho + row, tag, fadd(c.hs[row], y));
          } else if (PH == ST_DOWN) {
            const float v = fadd(c.hs[row], y);
            st_tag(a.t_hd + row, tag, v);
            if (last_layer) a.h_out[row] = v;
          } else {  // ST_HEAD
            a.logits[row] = y;
            if (am_better(y, row, best_v, best_i)) {
              best_v = y;
              best_i = row;
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&c.empty[slot]);
    c.pi++;
    if (flags & ST_LAST) break;
  }
  if (PH == ST_HEAD && lane == 0) {
    *best_out = best_v;
    *besti_out = best_i;
  }
  return true;
}

// Attention shared-memory layout (floats, inside the x region).
constexpr int SA_QRAW = 0, SA_KRAW = SA_QRAW + ST_MAX_G * 128, SA_VRAW = SA_KRAW + 128,
              SA_GQ = SA_VRAW + 128, SA_GK = SA_GQ + 128, SA_INV = SA_GK + 128,
              SA_QV = SA_INV + 64, SA_KNEW = SA_QV + ST_MAX_G * 128, SA_VNEW = SA_KNEW + 128,
              SA_SC = SA_VNEW + 128, SA_ML = SA_SC + ST_MAX_G * ST_KT,
              SA_CW = SA_ML + 4 * ST_MAX_G, SA_CL = SA_CW + ST_MAX_G * ST_MAX_SPLITS,
              SA_KT = SA_CL + 4 * ST_MAX_G, SA_KSTR = 132, SA_VT = SA_KT + ST_KT * SA_KSTR,
              SA_END = SA_VT + ST_KT * 128;

// Split count for a step over n_keys keys: one per ST_KT keys, at most
// splits_max (then each split walks several tiles).
FLOCK_DEV int st_splits(int n_keys, int splits_max) {
  const int s = (n_keys + ST_KT - 1) / ST_KT;
  return s < 1 ? 1 : (s > splits_max ? splits_max : s);
}

// K/V rows of keys [t0, t0 + nt) of kv head g (except key pos, not written
// yet) into registers: a tile is ST_KT x 128 floats = 1024 float4 per
// matrix, thread t holds float4 e = t + ST_CTHREADS * u; bf16 is widened.
constexpr int ST_TILE_F4 = ST_KT * 32;
constexpr int ST_TILE_PER = (ST_TILE_F4 + ST_CTHREADS - 1) / ST_CTHREADS;
struct StTile {
  float4 k[ST_TILE_PER], v[ST_TILE_PER];
};
FLOCK_DEV void st_tile_load(const StArgs& a, const StLayer& L, int g, int t0, int nt, int pos,
                            StTile& tl) {
  const int t = threadIdx.x;
  const size_t kvs = (size_t)a.nKV * a.hd;
#pragma unroll
  for (int u = 0; u < ST_TILE_PER; u++) {
    const int e = t + u * ST_CTHREADS;  // float4 index in the tile
    const int j = e >> 5, c4 = e & 31, key = t0 + j;
    float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk;
    if (e < ST_TILE_F4 && j < nt && key != pos) {
      const size_t off = (size_t)key * kvs + (size_t)g * 128;
      if (a.kv_bf16) {
        const uint2 kw = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(L.kcache) + off)[c4];
        const uint2 vw = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(L.vcache) + off)[c4];
        const float2 k0 = bf16x2_widen(kw.x), k1 = bf16x2_widen(kw.y);
        const float2 v0 = bf16x2_widen(vw.x), v1 = bf16x2_widen(vw.y);
        kk = make_float4(k0.x, k0.y, k1.x, k1.y);
        vv = make_float4(v0.x, v0.y, v1.x, v1.y);
      } else {
        kk = __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(L.kcache) + off) + c4);
        vv = __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(L.vcache) + off) + c4);
      }
    }
    tl.k[u] = kk;
    tl.v[u] = vv;
  }
}
FLOCK_DEV void st_tile_store(const StTile& tl, float* xs) {
  const int t = threadIdx.x;
#pragma unroll
  for (int u = 0; u < ST_TILE_PER; u++) {
    const int e = t + u * ST_CTHREADS;
    if (e >= ST_TILE_F4) break;
    const int j = e >> 5, c4 = e & 31;
    reinterpret_cast<float4*>(xs + SA_KT + j * SA_KSTR)[c4] = tl.k[u];
    reinterpret_cast<float4*>(xs + SA_VT)[e] = tl.v[u];
  }
}

// One attention item (kv head g, split s of S) for the token at pos; writes
// the partial (S > 1) or the output (S == 1); split 0 of S > 1 combines.
__device__ __noinline__ bool st_attention_item(const StArgs& a, const StLayer& L, StCta& c,
                                              int g, int s, int S, int pos, uint32_t tag) {
  const int G = a.nH / a.nKV;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float* xs = c.xs;
  const int n_keys = pos + 1;
  const int chunk = (n_keys + S - 1) / S;
  const int k0 = s * chunk, k1 = min(n_keys, k0 + chunk);
  const size_t kvs = (size_t)a.nKV * a.hd;
  bool ok = true;

  // the first tile's loads and the constant gains go out before the wait
  StTile tl;
  st_tile_load(a, L, g, k0, min(ST_KT, k1 - k0), pos, tl);
  if (t < 32) {
    reinterpret_cast<float4*>(xs + SA_GQ)[t] = reinterpret_cast<const float4*>(L.q_norm)[t];
    reinterpret_cast<float4*>(xs + SA_GK)[t] = reinterpret_cast<const float4*>(L.k_norm)[t];
    if (t < 16) reinterpret_cast<float4*>(xs + SA_INV)[t] = reinterpret_cast<const float4*>(a.inv_freq)[t];
  }
  // q heads g*G .. g*G+G-1, k head g, v head g of the QKV output
  {
    const int nq = G * 128;
    const int qoff = g * G * 128, koff = a.nH * 128 + g * 128, voff = koff + a.nKV * 128;
    // word pairs: q [0, nq/2), k [nq/2, nq/2 + 64), v [.. + 64)
    const int npairs = nq / 2 + 128;
    for (int i = t; i < npairs; i += ST_CTHREADS) {
      const uint64_t* src;
      float* dst;
      if (i < nq / 2) {
        src = a.t_qkv + qoff + 2 * i;
        dst = xs + SA_QRAW + 2 * i;
      } else if (i < nq / 2 + 64) {
        src = a.t_qkv + koff + 2 * (i - nq / 2);
        dst = xs + SA_KRAW + 2 * (i - nq / 2);
      } else {
        src = a.t_qkv + voff + 2 * (i - nq / 2 - 64);
        dst = xs + SA_VRAW + 2 * (i - nq / 2 - 64);
      }
      ulonglong2 w = st_ld2(src);
      if (ok && !st_wait2(src, tag, w, a.err)) {
        atomicExch(a.err, ST_ERR_DATA);
        ok = false;
      }
      dst[0] = val_of(w.x);
      dst[1] = val_of(w.y);
    }
  }
  st_tile_store(tl, xs);
  if (st_any(!ok)) return false;
  // exact per-head RMSNorm + RoPE (k_qk_norm_rope_append's arithmetic)
  float* qv = xs + SA_QV;
  float* knew = xs + SA_KNEW;
  float* vnew = xs + SA_VNEW;
  if (warp < G)
    norm_rope_warp(xs + SA_QRAW + warp * 128, xs + SA_GQ, a.eps, pos, xs + SA_INV, a.neox,
                   qv + warp * 128, lane);
  else if (warp == G)
    norm_rope_warp(xs + SA_KRAW, xs + SA_GK, a.eps, pos, xs + SA_INV, a.neox, knew, lane);
  else if (warp == G + 1)
    for (int i = lane; i < 128; i += 32) vnew[i] = xs[SA_VRAW + i];
  st_bar();
  const bool has_new = pos >= k0 && pos < k1;
  if (t < 128) {
    const size_t off = (size_t)pos * kvs + (size_t)g * 128 + t;
    if (a.kv_bf16) {
      // the cache keeps bf16: this step's scores use the rounded value too
      const uint16_t kb = bf16_bits(knew[t]), vb = bf16_bits(vnew[t]);
      knew[t] = __uint_as_float((uint32_t)kb << 16);
      vnew[t] = __uint_as_float((uint32_t)vb << 16);
      if (has_new) {
        static_cast<uint16_t*>(L.kcache)[off] = kb;
        static_cast<uint16_t*>(L.vcache)[off] = vb;
      }
    } else if (has_new) {
      static_cast<float*>(L.kcache)[off] = knew[t];
      static_cast<float*>(L.vcache)[off] = vnew[t];
    }
  }
  st_bar();

  const float scale = __double2float_rn(1.0 / sqrt((double)a.hd));
  float* sc = xs + SA_SC;
  float* ml = xs + SA_ML;  // per head: m, l, correction
  float* kt = xs + SA_KT;
  float* vt = xs + SA_VT;
  if (t < G) {
    ml[4 * t] = -INFINITY;
    ml[4 * t + 1] = 0.0f;
  }
  // outputs (hq, i) = oi / 128, oi % 128 for oi = t + ST_CTHREADS * u
  constexpr int OPER = (ST_MAX_G * 128 + ST_CTHREADS - 1) / ST_CTHREADS;
  float o[OPER];
#pragma unroll
  for (int u = 0; u < OPER; u++) o[u] = 0.0f;
  for (int t0 = k0; t0 < k1; t0 += ST_KT) {
    const int nt = min(ST_KT, k1 - t0);
    if (t0 != k0) {
      st_bar();
      st_tile_load(a, L, g, t0, nt, pos, tl);
      st_tile_store(tl, xs);
    }
    if (pos >= t0 && pos < t0 + nt && t < 128) {
      kt[(pos - t0) * SA_KSTR + t] = knew[t];
      vt[(pos - t0) * 128 + t] = vnew[t];
    }
    st_bar();
    // scores: 4 threads per (query head, key), 32 dims each; lane = key low
    // 3 bits + 8 * quarter, so a quarter-warp reads 8 distinct K rows
    for (int u = t; u < G * ST_KT * 4; u += ST_CTHREADS) {
      const int w = u >> 5, ln = u & 31;
      const int quarter = ln >> 3;
      const int hq = w / (ST_KT / 8), j = (w % (ST_KT / 8)) * 8 + (ln & 7);
      float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f, p3 = 0.0f;
      if (j < nt) {
        const float4* kr = reinterpret_cast<const float4*>(kt + j * SA_KSTR + quarter * 32);
        const float4* qr = reinterpret_cast<const float4*>(qv + hq * 128 + quarter * 32);
#pragma unroll
        for (int c4 = 0; c4 < 8; c4++) {
          const float4 kk = kr[c4], qq = qr[c4];
          p0 = fmaf(qq.x, kk.x, p0);
          p1 = fmaf(qq.y, kk.y, p1);
          p2 = fmaf(qq.z, kk.z, p2);
          p3 = fmaf(qq.w, kk.w, p3);
        }
      }
      float d = (p0 + p1) + (p2 + p3);
      d += __shfl_xor_sync(0xffffffffu, d, 8);
      d += __shfl_xor_sync(0xffffffffu, d, 16);
      if (quarter == 0 && j < nt) sc[hq * ST_KT + j] = d * scale;
    }
    st_bar();
    if (warp < G) {
      const int hq = warp;
      const float v = lane < nt ? sc[hq * ST_KT + lane] : -INFINITY;
      float mt = v;
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o2));
      const float m_old = ml[4 * hq];
      const float m_new = fmaxf(m_old, mt);
      const float p = lane < nt ? expf(v - m_new) : 0.0f;
      if (lane < nt) sc[hq * ST_KT + lane] = p;
      float lt = p;
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o2);
      if (lane == 0) {
        const float cr = expf(m_old - m_new);
        ml[4 * hq] = m_new;
        ml[4 * hq + 1] = fmaf(ml[4 * hq + 1], cr, lt);
        ml[4 * hq + 2] = cr;
      }
    }
    st_bar();
#pragma unroll
    for (int u = 0; u < OPER; u++) {
      const int oi = t + u * ST_CTHREADS;
      if (oi < G * 128) {
        const int hq = oi >> 7, i = oi & 127;
        float acc = o[u] * ml[4 * hq + 2];
        for (int j = 0; j < nt; j++) acc = fmaf(sc[hq * ST_KT + j], vt[j * 128 + i], acc);
        o[u] = acc;
      }
    }
  }
  if (S == 1) {
#pragma unroll
    for (int u = 0; u < OPER; u++) {
      const int oi = t + u * ST_CTHREADS;
      if (oi < G * 128)
        st_tag(a.t_att + (size_t)g * G * 128 + oi, tag, o[u] / ml[4 * (oi >> 7) + 1]);
    }
    return true;
  }
  // this split's partial
  if (s > 0) {
#pragma unroll
    for (int u = 0; u < OPER; u++) {
      const int oi = t + u * ST_CTHREADS;
      if (oi < G * 128) {
        const int hq = oi >> 7, i = oi & 127;
        uint64_t* pp = a.t_part + ((size_t)(g * G + hq) * ST_MAX_SPLITS + s) * ST_PSTRIDE;
        st_tag(pp + i, tag, o[u]);
        if (i == 0) {
          st_tag(pp + 128, tag, ml[4 * hq]);
          st_tag(pp + 129, tag, ml[4 * hq + 1]);
        }
      }
    }
    return true;
  }
  // split 0 combines: warp hq derives head hq's split weights w_s = e^(m_s -
  // M) and L = sum l_s w_s (lane s holds splits s, s + 32); then every thread
  // sums its element over the splits in order, 16 loads in flight at a time
  float* cw = xs + SA_CW;
  float* cl = xs + SA_CL;
  if (warp < G) {
    const uint64_t* pp = a.t_part + (size_t)(g * G + warp) * ST_MAX_SPLITS * ST_PSTRIDE;
    float mv[2], lv[2];
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int sp = lane + 32 * u;
      mv[u] = -INFINITY;
      lv[u] = 0.0f;
      if (sp == 0) {
        mv[u] = ml[4 * warp];
        lv[u] = ml[4 * warp + 1];
      } else if (sp < S) {
        ulonglong2 w = st_ld2(pp + (size_t)sp * ST_PSTRIDE + 128);
        if (ok && !st_wait2(pp + (size_t)sp * ST_PSTRIDE + 128, tag, w, a.err)) {
          atomicExch(a.err, ST_ERR_DATA);
          ok = false;
        }
        mv[u] = val_of(w.x);
        lv[u] = val_of(w.y);
      }
    }
    float M = fmaxf(mv[0], mv[1]);
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
    const float w0 = lane < S ? expf(mv[0] - M) : 0.0f;
    const float w1 = lane + 32 < S ? expf(mv[1] - M) : 0.0f;
    float Lsum = 0.0f;
    for (int sp = 0; sp < S; sp++) {
      const bool hi = sp >= 32;
      Lsum = fmaf(__shfl_sync(0xffffffffu, hi ? lv[1] : lv[0], sp & 31),
                  __shfl_sync(0xffffffffu, hi ? w1 : w0, sp & 31), Lsum);
    }
    cw[warp * ST_MAX_SPLITS + lane] = w0;
    cw[warp * ST_MAX_SPLITS + lane + 32] = w1;
    if (lane == 0) cl[warp] = Lsum;
  }
  st_bar();
#pragma unroll
  for (int u = 0; u < OPER; u++) {
    const int oi = t + u * ST_CTHREADS;
    if (oi >= G * 128) break;
    const int hq = oi >> 7, i = oi & 127;
    const uint64_t* pp = a.t_part + (size_t)(g * G + hq) * ST_MAX_SPLITS * ST_PSTRIDE + i;
    float O = fmaf(o[u], cw[hq * ST_MAX_SPLITS], 0.0f);
    for (int s0 = 1; s0 < S; s0 += 16) {
      uint64_t w[16];
#pragma unroll
      for (int u = 0; u < 16; u++)
        if (s0 + u < S) w[u] = st_ld1(pp + (size_t)(s0 + u) * ST_PSTRIDE);
#pragma unroll
      for (int u = 0; u < 16; u++) {
        if (s0 + u >= S) break;
        if (ok && !st_wait1(pp + (size_t)(s0 + u) * ST_PSTRIDE, tag, w[u], a.err)) {
          atomicExch(a.err, ST_ERR_DATA);
          ok = false;
        }
        O = fmaf(val_of(w[u]), cw[hq * ST_MAX_SPLITS + s0 + u], O);
      }
    }
    st_tag(a.t_att + (size_t)(g * G + hq) * 128 + i, tag, O / cl[hq]);
  }
  return ok;
}

// The producer warp: stream this CTA's pieces into the ring in order.
__device__ __noinline__ void st_producer(const StArgs& a, StCta& c) {
  const int lane = threadIdx.x & 31;
  const StPiece* P = a.pieces + (size_t)blockIdx.x * a.max_pieces;
  const int np = a.n_pieces[blockIdx.x];
  int issued = 0;
  bool fail = false;
  for (int base = 0; base < np && !fail; base += 32) {
    uint4 d0 = make_uint4(0, 0, 0, 0), d1 = d0, d2 = d0;
    if (base + lane < np) {
      const uint4* src = reinterpret_cast<const uint4*>(P + base + lane);
      d0 = __ldg(src);
      d1 = __ldg(src + 1);
      d2 = __ldg(src + 2);
    }
    const int nb = min(32, np - base);
    for (int j = 0; j < nb; j++) {
      uint32_t w[12] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w, d2.x, d2.y, d2.z, d2.w};
#pragma unroll
      for (int q = 0; q < 12; q++) w[q] = __shfl_sync(0xffffffffu, w[q], j);
      const int i = base + j;
      const int slot = i % a.ring_slots;
      const uint32_t round = (uint32_t)(i / a.ring_slots);
      if (lane == 0) {
        if (round > 0 && !mbar_wait(&c.empty[slot], (round - 1) & 1u, a.err)) {
          fail = true;
        } else {
          uint4* h = reinterpret_cast<uint4*>(&c.hdr[slot]);
          h[0] = make_uint4(w[0], w[1], w[2], w[3]);
          h[1] = make_uint4(w[4], w[5], w[6], w[7]);
          h[2] = make_uint4(w[8], w[9], w[10], w[11]);
          const StPiece& p = c.hdr[slot];
          const int nsub = (p.flags & ST_PAIR) ? 2 : 1;
          const uint32_t bytes = p.nrows ? nsub * (p.qs_bytes + p.sc_bytes) : 0u;
          mbar_expect_tx(&c.full[slot], bytes);
          if (p.nrows) {
            uint8_t* dst = c.ring + (size_t)slot * ST_SLOT;
            for (int u = 0; u < nsub; u++) {
              bulk_g2s(dst, p.qs[u], p.qs_bytes, &c.full[slot]);
              bulk_g2s(dst + p.qs_bytes, p.sc[u], p.sc_bytes, &c.full[slot]);
              dst += p.qs_bytes + p.sc_bytes;
            }
          }
          issued = i + 1;
        }
      }
      fail = __shfl_sync(0xffffffffu, fail ? 1 : 0, 0) != 0;
      if (fail) break;
    }
  }
  if (lane == 0) {
    c.flags[0] = issued;
    if (fail) atomicExch(a.err, ST_ERR_RING);
  }
}

static __global__ void __launch_bounds__(ST_THREADS, 1) k_decode_stream(const StArgs a) {
  extern __shared__ __align__(1024) uint8_t st_smem[];
  StCta c;
  c.ring = st_smem;
  c.hdr = reinterpret_cast<StPiece*>(st_smem + (size_t)a.ring_slots * ST_SLOT);
  c.full = reinterpret_cast<uint64_t*>(c.hdr + a.ring_slots);
  c.empty = c.full + a.ring_slots;
  c.xs = reinterpret_cast<float*>(c.empty + a.ring_slots);
  c.hs = c.xs + a.xbytes / 4;
  c.gs = c.hs + a.H;
  c.red = c.gs + max(a.H, a.F);
  c.am_v = c.red + 136;
  c.am_i = reinterpret_cast<uint32_t*>(c.am_v + ST_CWARPS);
  c.flags = reinterpret_cast<int*>(c.am_i + ST_CWARPS);
  c.pi = 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.ring_slots; i++) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], ST_CWARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    c.flags[0] = 0;
    c.flags[1] = 0;
  }
  __syncthreads();

  if (warp == ST_CWARPS) {
    st_producer(a, c);
  } else {
    unsigned long long* tr =
        a.trace ? a.trace + (size_t)blockIdx.x * st_trace_stride(a.n_layers) : nullptr;
    auto stamp = [&](int i) {
      if (tr && threadIdx.x == 0) tr[i] = globaltimer_ns();
    };
    stamp(0);
    const int pos = a.ctl[0] + a.ctl[1];
    const int token = a.ids[0];
    const uint32_t seq = *a.seq;
    const int t = threadIdx.x;
    const int S = st_splits(pos + 1, a.splits_max);
    const int n_items = a.nKV * S;
    // layer 0's input: the embedded token (k_embed's arithmetic), computed
    // by every CTA
    for (int q = t; q < a.H / 4; q += ST_CTHREADS) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (token >= 0 && token < a.vocab) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(a.embd_qs + (size_t)token * a.H + 4 * q);
        const float sc = scale_f16(a.embd_sc[(size_t)token * a.embd_sc_stride + q / 8]);
        float q0, q1, q2, q3;
        dec_i8x4(w, q0, q1, q2, q3);
        v = make_float4(fmul(q0, sc), fmul(q1, sc), fmul(q2, sc), fmul(q3, sc));
      }
      reinterpret_cast<float4*>(c.hs)[q] = v;
    }
    float best_v = -FLT_MAX;
    uint32_t best_i = 0xFFFFFFFFu;
    const int nbH = a.H / 32;
    const bool xregH = nbH <= 32;
    // every fallible step ends in st_any, so `ok` is uniform over the CTA
    bool ok = true;
    for (int l = 0; l < a.n_layers; l++) {
      const StLayer& L = a.layers[l];
      const uint32_t tag = (seq << 8) | (uint32_t)l;
      const bool last = l == a.n_layers - 1;
      // ---- QKV: x = rmsnorm(h, attn_norm); h = the last down's output (the
      // previous iteration ended in st_any: its epilogues are done with hs)
      for (int i = t; i < a.H; i += ST_CTHREADS) c.gs[i] = __ldg(L.attn_norm + i);
      if (l > 0) ok = st_poll_vec<false>(a.t_hd, a.H, tag - 1, c.hs, a.err);
      if (st_any(!ok)) break;
      st_rmsnorm(c.hs, c.gs, a.H, a.eps, c.xs, c.red);
      ok = xregH ? st_phase<ST_QKV, true>(a, c, tag, last, &best_v, &best_i)
                 : st_phase<ST_QKV, false>(a, c, tag, last, &best_v, &best_i);
      stamp(1 + 6 * l);
      if (st_any(!ok)) break;  // also: every warp is done with xs
      // ---- attention items of this CTA (at most one: items <= grid)
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        ok = st_attention_item(a, L, c, item / S, item % S, S, pos, tag);
        if (st_any(!ok)) break;
      }
      stamp(2 + 6 * l);
      if (!ok) break;
      // ---- o_proj + residual: x = attention output
      ok = st_poll_vec<true>(a.t_att, a.nH * a.hd, tag, c.xs, a.err);
      if (st_any(!ok)) break;
      ok = st_phase<ST_O, false>(a, c, tag, last, &best_v, &best_i);
      stamp(3 + 6 * l);
      if (st_any(!ok)) break;  // also: every warp is done with hs and xs
      // ---- gate/up + SwiGLU: x = rmsnorm(h, ffn_norm)
      for (int i = t; i < a.H; i += ST_CTHREADS) c.gs[i] = __ldg(L.ffn_norm + i);
      ok = st_poll_vec<false>(a.t_ho, a.H, tag, c.hs, a.err);
      if (st_any(!ok)) break;
      st_rmsnorm(c.hs, c.gs, a.H, a.eps, c.xs, c.red);
      ok = xregH ? st_phase<ST_GU, true>(a, c, tag, last, &best_v, &best_i)
                 : st_phase<ST_GU, false>(a, c, tag, last, &best_v, &best_i);
      stamp(4 + 6 * l);
      if (st_any(!ok)) break;  // also: every warp is done with xs
      // ---- down + residual: x = act
      ok = st_poll_vec<true>(a.t_act, a.F, tag, c.xs, a.err);
      if (st_any(!ok)) break;
      ok = st_phase<ST_DOWN, false>(a, c, tag, last, &best_v, &best_i);
      stamp(5 + 6 * l);
      if (st_any(!ok)) break;
    }
    if (ok) {
      // ---- output_norm + head + argmax (hs is free: the loop ended in st_any)
      const uint32_t tag = (seq << 8) | (uint32_t)(a.n_layers - 1);
      for (int i = t; i < a.H; i += ST_CTHREADS) c.gs[i] = __ldg(a.out_norm + i);
      ok = st_poll_vec<false>(a.t_hd, a.H, tag, c.hs, a.err);
      if (!st_any(!ok)) {
        st_rmsnorm(c.hs, c.gs, a.H, a.eps, c.xs, c.red);
        ok = xregH ? st_phase<ST_HEAD, true>(a, c, tag, true, &best_v, &best_i)
                   : st_phase<ST_HEAD, false>(a, c, tag, true, &best_v, &best_i);
      }
      stamp(2 + 6 * a.n_layers);
    }
    // CTA argmax, then the last CTA reduces the grid's (kernels/argmax.wgsl
    // pass 1 / pass 2; lowest index on ties)
    if (lane == 0) {
      c.am_v[warp] = best_v;
      c.am_i[warp] = best_i;
    }
    st_bar();
    if (t == 0) {
      float bv = c.am_v[0];
      uint32_t bi = c.am_i[0];
      for (int w = 1; w < ST_CWARPS; w++)
        if (am_better(c.am_v[w], c.am_i[w], bv, bi)) {
          bv = c.am_v[w];
          bi = c.am_i[w];
        }
      a.am_val[blockIdx.x] = bv;
      a.am_idx[blockIdx.x] = bi;
      __threadfence();
      const uint32_t prev = atomicAdd(a.am_count, 1u);
      c.flags[1] = prev == gridDim.x - 1;
    }
    st_bar();
    if (c.flags[1]) {
      __threadfence();
      float bv = -FLT_MAX;
      uint32_t bi = 0xFFFFFFFFu;
      for (int i = t; i < (int)gridDim.x; i += ST_CTHREADS) {
        const float v = ((volatile float*)a.am_val)[i];
        const uint32_t ix = ((volatile uint32_t*)a.am_idx)[i];
        if (am_better(v, ix, bv, bi)) {
          bv = v;
          bi = ix;
        }
      }
#pragma unroll
      for (int s2 = 16; s2 > 0; s2 >>= 1) {
        const float ov = __shfl_down_sync(0xffffffffu, bv, s2);
        const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, s2);
        if (am_better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        c.am_v[warp] = bv;
        c.am_i[warp] = bi;
      }
      st_bar();
      if (t == 0) {
        bv = c.am_v[0];
        bi = c.am_i[0];
        for (int w = 1; w < ST_CWARPS; w++)
          if (am_better(c.am_v[w], c.am_i[w], bv, bi)) {
            bv = c.am_v[w];
            bi = c.am_i[w];
          }
        if (!*(volatile int*)a.err) {
          a.ids[0] = (int32_t)bi;
          if (pos >= 0 && pos < a.hist_cap) a.hist[pos] = (int32_t)bi;
          a.ctl[0] = pos;
          a.ctl[1] = 1;
        }
        // next launch's tags; 24 bits of sequence, never 0
        *a.seq = (seq % 0xFFFFFEu) + 1u;
        *a.am_count = 0;
      }
    }
    stamp(3 + 6 * a.n_layers);
  }
  __syncthreads();
  // every bulk copy issued must land before the CTA exits: wait (bounded)
  // for the slots of pieces issued but not consumed (only after an error)
  if (threadIdx.x == 0) {
    const int issued = c.flags[0];
    for (int i = c.pi; i < issued; i++) {
      const int slot = i % a.ring_slots;
      mbar_wait(&c.full[slot], (uint32_t)(i / a.ring_slots) & 1u, a.err, false);
    }
  }
}

// Dynamic shared memory of a k_decode_stream launch with `slots` ring slots.
inline size_t st_fixed_bytes(int H, int qw, int F, int* xbytes) {
  const int kmax = H > qw ? (H > F ? H : F) : (qw > F ? qw : F);
  const size_t xs = (size_t)kmax / 32 * XPAD * 4;
  const size_t at = (size_t)SA_END * 4;
  const size_t xb = ((xs > at ? xs : at) + 15) / 16 * 16;
  *xbytes = (int)xb;
  const int hf = H > F ? H : F;
  return xb + (size_t)H * 4 + (size_t)hf * 4 + 136 * 4 + ST_CWARPS * 8 + 16;
}
inline size_t st_smem_bytes(int slots, size_t fixed) {
  return (size_t)slots * (ST_SLOT + sizeof(StPiece) + 16) + fixed;
}

}  // namespace flock
