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
//    pieces, in the order they are consumed, into a ring of 17 KiB
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

// 8 compute warps + the producer warp: 9 warps leave a thread up to 168
// registers (three warps per SM sub-partition).  With 15 compute warps (128
// registers) the whole kernel spilled inside its row loops -- local memory
// costs an L2 round trip here, L1 being almost all shared memory -- and
// measured slower, though the loop alone is faster with more warps.
constexpr int ST_CWARPS = 8;
constexpr int ST_CTHREADS = ST_CWARPS * 32;
constexpr int ST_THREADS = ST_CTHREADS + 32;  // + the producer warp
// bytes per ring slot: 16 rows of K = 1024 (1088 B with scales), 8 of 2048,
// 4 of 4096, 8 gate/up pairs of 1024 -- multiples of the 8 compute warps
constexpr int ST_SLOT = 17408;
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
  uint32_t row_bytes;  // K: int8 weights per row
  uint32_t out_row;
  uint16_t sc_row;     // scale bytes per row (sc_stride * 2)
  uint16_t nrows;
  uint16_t flags;
  uint16_t pad;
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
  // RoPE (cos, sin) per position and frequency, [rope_rows][hd / 2]: the
  // values norm_rope_warp computes (f64 cos/sin of fr(pos * inv_freq[i])
  // rounded once), tabulated when the engine is built
  const float2* rope_cs;
  int rope_rows;
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
  int head;       // 1: the LM head and its argmax run in this kernel; 0: a GEMV launch follows
  int l2_rounds;  // producer lanes prefetch into L2 the piece this many ring rounds ahead
  int ring_slots;
  int xbytes;  // bytes of the x-staging / attention union region
};

// Phase trace (optional, per CTA; global-timer ns): [0] start, [1] embedded;
// per layer l at 2 + 10 l: h polled, QKV rows done, q/k/v polled (attention
// CTAs, else 0), attention done, attention output polled, o_proj rows done,
// h polled, gate/up rows done, act polled, down rows done; then head input
// polled, head rows done, finish, the consumer's total ns waiting for ring
// slots to fill, the producer's total ns waiting for slots to drain, and the
// pieces issued.
// Then 12 words of the last layer's attention item, on the CTAs that run
// one: q/k/v polled, q/k rotated, new key appended, tile staged, scores,
// softmax, P.V, partial published / combine weights, combined.
// Then 27 words: the last layer's QKV, gate/up and down phases, 9 each --
// start, then for up to 4 pieces "ring slot full" and "rows done".
__host__ __device__ inline int st_trace_stride(int n_layers) { return 47 + 10 * n_layers; }

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
    if (i >= 32) __nanosleep(20);  // the first polls spin: a miss costs one L2 round trip
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
    if (i >= 32) __nanosleep(20);  // the first polls spin: a miss costs one L2 round trip
    w = st_ld1(p);
  }
  return true;
}

// The n tagged words at src into dst (packed: the Q8_0 packed-pair x layout
// of the folds; else plain), waiting for tag.  All of a thread's loads are
// issued before any is checked.  Called by the compute threads; false (and
// *err set) on a timeout.
FLOCK_DEV bool st_poll_vec(const uint64_t* src, int n, uint32_t tag, float* dst, bool packed,
                           int* err) {
  // up to ST_POLL pairs a thread, all loads issued before the first is
  // checked: a vector lands in one L2 round trip, not one per pair
  constexpr int ST_POLL = 6;
  const int t = threadIdx.x;
  const int np = n / 2;
  bool ok = true;
  for (int base = 0; base < np; base += ST_POLL * ST_CTHREADS) {
    ulonglong2 w[ST_POLL];
#pragma unroll
    for (int u = 0; u < ST_POLL; u++) {
      const int i = base + t + u * ST_CTHREADS;
      if (i < np) w[u] = st_ld2(src + 2 * i);
    }
#pragma unroll
    for (int u = 0; u < ST_POLL; u++) {
      const int i = base + t + u * ST_CTHREADS;
      if (i >= np) continue;
      if (ok && !st_wait2(src + 2 * i, tag, w[u], err)) {
        ok = false;
        atomicExch(err, ST_ERR_DATA);
      }
      const int e = 2 * i;
      dst[packed ? xperm<QT_Q8>(e) : e] = val_of(w[u].x);
      dst[packed ? xperm<QT_Q8>(e + 1) : e + 1] = val_of(w[u].y);
    }
  }
  return ok;
}

// ops_ref.ts:20 rmsnormRef with WG = 128 (rmsnorm_to_smem's arithmetic):
// src plain [n] in shared memory, gain staged in gs, result in xs in the
// packed-pair layout.  Called by the compute threads after a barrier that
// made src and gs visible; ends with a barrier.
FLOCK_DEV void st_rmsnorm(const float* src, const float* gs, int n, float eps, float* xs,
                          float* red) {
  const int t = threadIdx.x, lane = t & 31;
  if (t < 32) {
    // warp 0 holds partials t = lane + 32q: the 128-wide tree's first two
    // levels (t + 64, then t + 32) are lane-local, the rest is the warp tree
    float p[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      float acc = 0.0f;
      for (int i = lane + 32 * q; i < n; i += 128) acc = ffma(src[i], src[i], acc);
      p[q] = acc;
    }
    float v = fadd(fadd(p[0], p[2]), fadd(p[1], p[3]));
    v = warp_tree_sum(v);
    if (lane == 0) red[128] = rsqrt_f64r(fadd(fdiv(v, (float)n), eps));
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

// Shared-memory regions of one CTA, computed from the arguments (a few
// integer ops) wherever they are needed: passing a struct of them by
// reference to the out-of-line phases would put it in local memory, which
// with almost all of L1 given to shared memory lives in L2.
struct StCta {
  uint8_t* ring;
  StPiece* hdr;
  uint64_t* full;
  uint64_t* empty;
  float* xs;   // x staging (packed) | attention tiles
  float* hs;   // [H] plain: the residual stream as this CTA last read it
  float* gs;   // [max(H, F)] gains staging
  float* red;  // [136]
  float* split;  // [ST_CWARPS][32] lane accumulators of split rows
  float* am_v; // [ST_CWARPS]
  uint32_t* am_i;
  int* flags;  // [0]: pieces issued (producer), [1]: last-CTA flag, [2]: pos,
               // [3]: launch sequence, [4]: attention splits, [8 + s]: the first
               // piece of ring slot s not issued
  unsigned long long* wait_ns;  // trace: compute thread 0's time waiting for slots to fill
};

FLOCK_DEV StCta st_cta(const StArgs& a) {
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
  c.split = c.red + 136;
  c.am_v = c.split + ST_CWARPS * 32;
  c.am_i = reinterpret_cast<uint32_t*>(c.am_v + ST_CWARPS);
  c.wait_ns = reinterpret_cast<unsigned long long*>(c.am_i + ST_CWARPS);
  c.flags = reinterpret_cast<int*>(c.wait_ns + 1);
  return c;
}

enum { ST_QKV = 0, ST_O = 1, ST_GU = 2, ST_DOWN = 3, ST_HEAD = 4 };

// The rows of one phase: every piece up to and including the ST_LAST one.
// EPI by phase: QKV -> tagged q|k|v; O / DOWN -> tagged h = hs[row] + y
// (DOWN of the last layer also writes h_out); GU -> tagged SwiGLU(gate, up);
// HEAD -> logits and this warp's argmax (best_v / best_i in lane 0).
// Half of a long row (K > 1024): the blocks lane + 32m with m of parity h,
// folded in gemv_run's order into one logical lane's accumulator.
FLOCK_DEV float st_half(const uint8_t* q, const uint16_t* s, int nb, const float* xs, int h,
                        int lane) {
  float acc = 0.0f;
  const int M = (nb + 31) / 32;
#pragma unroll 1
  for (int m = h; m < M; m += 2) {
    const int b = lane + 32 * m;
    if (b >= nb) break;
    BlockW<QT_Q8> bw;
    bw.w0 = *reinterpret_cast<const uint4*>(q + b * 32);
    bw.w1 = *reinterpret_cast<const uint4*>(q + b * 32 + 16);
    bw.s = s[b];
    uint64_t xq[16];
    load_pairs(xs, b, xq);
    acc = fold_block_packed<QT_Q8>(bw, xq, acc);
  }
  return acc;
}

// One row's epilogue (lane 0 of the warp holding y).
FLOCK_DEV void st_epilogue(int ph, uint64_t* out, const float* hs, float* h_out, float* logits,
                           uint32_t tag, bool last_layer, uint32_t row, float y, float u,
                           float& best_v, uint32_t& best_i) {
  if (ph == ST_GU) {
    // ops_ref.ts:103 swigluRef: fr(fr(g / fr(1 + fr(exp(-g)))) * up)
    const float e = exp_f64r(-y);
    st_tag(out + row, tag, fmul(fdiv(y, fadd(1.0f, e)), u));
  } else if (ph == ST_QKV) {
    st_tag(out + row, tag, y);
  } else if (ph == ST_O) {
    st_tag(out + row, tag, fadd(hs[row], y));
  } else if (ph == ST_DOWN) {
    const float v = fadd(hs[row], y);
    st_tag(out + row, tag, v);
    if (last_layer) h_out[row] = v;
  } else {  // ST_HEAD
    logits[row] = y;
    if (am_better(y, row, best_v, best_i)) {
      best_v = y;
      best_i = row;
    }
  }
}

// The rows of one phase: every piece up to and including the ST_LAST one.
// Returns the next piece index, or -1 on a timeout.  HEAD leaves each warp's
// best (value, row) in the CTA's argmax slots.
//  * XREG (K <= 1024, one block per lane, x pairs in registers): a warp per
//    row (a gate/up pair: its two rows as independent chains);
//  * longer rows, when the piece has a row (pair) for every warp: a warp per
//    row, gemv_run's order;
//  * longer rows in a piece too small for that: a row is two items, its even
//    and odd blocks (logical lanes t and t + 32), folded by two warps; the
//    halves meet in shared memory and the warp of the even half finishes the
//    row -- fadd of the two lane accumulators, then the tree, exactly as
//    gemv_run.  One barrier round (every compute warp takes part, so the
//    ring wait is agreed on first).
template <bool XREG>
FLOCK_DEV int st_phase(const StArgs& a, int pi, int ph, uint32_t tag, bool last_layer,
                       unsigned long long* pd) {
  // everything the loop needs, read once: the loop's stores could alias the
  // argument reference, so reads through it would be repeated every row
  const StCta c = st_cta(a);
  const int ns = a.ring_slots;
  int* const err = a.err;
  const bool trace = a.trace != nullptr;
  uint64_t* const out = ph == ST_QKV ? a.t_qkv : ph == ST_O ? a.t_ho : ph == ST_GU ? a.t_act
                                                                                  : a.t_hd;
  float* const h_out = a.h_out;
  float* const logits = a.logits;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t xp[16];
  if (XREG) st_xregs(c.xs, a.H / 32, xp);
  float best_v = -FLT_MAX;
  uint32_t best_i = 0xFFFFFFFFu;
  pd = threadIdx.x == 0 ? pd : nullptr;
  if (pd) pd[0] = globaltimer_ns();
  for (int k = 0;; k++) {
    const int slot = pi % ns;
    const uint32_t par = (uint32_t)(pi / ns) & 1u;
    const uint64_t w0 = (trace && threadIdx.x == 0) ? globaltimer_ns() : 0;
    bool ok = mbar_wait_poll(&c.full[slot], par, err);
    if (!XREG) ok = !st_any(!ok);  // the split path meets barriers below
    if (!ok) {
      if (lane == 0) atomicExch(err, ST_ERR_RING);
      return -1;
    }
    if (w0) *c.wait_ns += globaltimer_ns() - w0;
    if (pd && k < 4) pd[1 + 2 * k] = globaltimer_ns();
    const StPiece& p = c.hdr[slot];
    const int n = p.nrows;
    const uint16_t flags = p.flags;
    const uint32_t out0 = p.out_row;
    if (n > 0) {
      const int K = (int)p.row_bytes;
      const int scs = p.sc_row >> 1;  // halfs per scale row
      const uint32_t qsb = (uint32_t)n * (uint32_t)K, scb = (uint32_t)n * p.sc_row;
      const int nb = K / 32;
      const uint8_t* qa = c.ring + (size_t)slot * ST_SLOT;
      const uint16_t* sa = reinterpret_cast<const uint16_t*>(qa + qsb);
      const uint8_t* qb = qa + qsb + scb;
      const uint16_t* sb = reinterpret_cast<const uint16_t*>(qb + qsb);
      if (XREG) {
        if (flags & ST_PAIR) {  // a gate/up pair per warp: two independent rows
          for (int r = warp; r < n; r += ST_CWARPS) {
            const float y = st_row<true>(qa + (size_t)r * K, sa + (size_t)r * scs, nb, c.xs, xp, lane);
            const float u = st_row<true>(qb + (size_t)r * K, sb + (size_t)r * scs, nb, c.xs, xp, lane);
            if (lane == 0)
              st_epilogue(ph, out, c.hs, h_out, logits, tag, last_layer, out0 + r, y, u, best_v,
                              best_i);
          }
        } else if (n <= ST_CWARPS) {  // a row per warp
          for (int r = warp; r < n; r += ST_CWARPS) {
            const float y = st_row<true>(qa + (size_t)r * K, sa + (size_t)r * scs, nb, c.xs, xp, lane);
            if (lane == 0)
              st_epilogue(ph, out, c.hs, h_out, logits, tag, last_layer, out0 + r, y, 0.0f, best_v,
                          best_i);
          }
        } else {  // rows r and r + ST_CWARPS together (the second may repeat the first)
          for (int r = warp; r < n; r += 2 * ST_CWARPS) {
            const bool two = r + ST_CWARPS < n;
            const int r2 = two ? r + ST_CWARPS : r;
            const float y = st_row<true>(qa + (size_t)r * K, sa + (size_t)r * scs, nb, c.xs, xp, lane);
            const float y2 = st_row<true>(qa + (size_t)r2 * K, sa + (size_t)r2 * scs, nb, c.xs, xp, lane);
            if (lane == 0) {
              st_epilogue(ph, out, c.hs, h_out, logits, tag, last_layer, out0 + r, y, 0.0f, best_v,
                              best_i);
              if (two)
                st_epilogue(ph, out, c.hs, h_out, logits, tag, last_layer, out0 + r2, y2, 0.0f,
                                best_v, best_i);
            }
          }
        }
      } else if (n * ((flags & ST_PAIR) ? 4 : 2) > ST_CWARPS) {
        // enough rows for every warp: a warp per row (pair), both halves
        for (int r = warp; r < n; r += ST_CWARPS) {
          const float y = st_row<false>(qa + (size_t)r * K, sa + (size_t)r * scs, nb, c.xs, xp, lane);
          const float u = (flags & ST_PAIR) ? st_row<false>(qb + (size_t)r * K, sb + (size_t)r * scs,
                                                            nb, c.xs, xp, lane)
                                            : 0.0f;
          if (lane == 0)
            st_epilogue(ph, out, c.hs, h_out, logits, tag, last_layer, out0 + r, y, u, best_v,
                            best_i);
        }
      } else {
        // items per row: (matrix, half) -- 2, or 4 for a gate/up pair
        const int IPR = (flags & ST_PAIR) ? 4 : 2;
        const int RPR = ST_CWARPS / IPR;  // rows per round
        float* half = c.split;                 // [ST_CWARPS][32] lane accumulators
        const int rw = warp / IPR, sub = (warp / 2) % (IPR / 2), h = warp & 1;
        for (int r0 = 0; r0 < n; r0 += RPR) {
          const int rr = r0 + rw;
          const bool mine = warp < IPR * RPR && rr < n;
          float acc = 0.0f;
          if (mine)
            acc = sub == 0 ? st_half(qa + (size_t)rr * K, sa + (size_t)rr * scs, nb, c.xs, h, lane)
                           : st_half(qb + (size_t)rr * K, sb + (size_t)rr * scs, nb, c.xs, h, lane);
          half[warp * 32 + lane] = acc;
          st_bar();
          if (mine && warp % IPR == 0) {
            const float y = warp_tree_sum(fadd(acc, half[(warp + 1) * 32 + lane]));
            const float u = IPR == 4 ? warp_tree_sum(fadd(half[(warp + 2) * 32 + lane],
                                                          half[(warp + 3) * 32 + lane]))
                                     : 0.0f;
            if (lane == 0)
              st_epilogue(ph, out, c.hs, h_out, logits, tag, last_layer, out0 + rr, y, u, best_v,
                              best_i);
          }
          st_bar();  // the scratch is reused by the next round
        }
      }
    }
    // order this lane's generic reads of the slot before the producer's next
    // bulk copy (async proxy) into it, then release the slot for the warp
    fence_proxy_async_smem();
    __syncwarp();
    if (pd && k < 4) pd[2 + 2 * k] = globaltimer_ns();
    if (lane == 0) mbar_arrive(&c.empty[slot]);
    pi++;
    if (flags & ST_LAST) break;
  }
  if (ph == ST_HEAD && lane == 0) {
    c.am_v[warp] = best_v;
    c.am_i[warp] = best_i;
  }
  return pi;
}

// Attention shared-memory layout (floats, inside the x region).
constexpr int SA_QRAW = 0, SA_KRAW = SA_QRAW + ST_MAX_G * 128, SA_VRAW = SA_KRAW + 128,
              SA_GQ = SA_VRAW + 128, SA_GK = SA_GQ + 128, SA_CS = SA_GK + 128,
              SA_QV = SA_CS + 128, SA_KNEW = SA_QV + ST_MAX_G * 128, SA_VNEW = SA_KNEW + 128,
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
FLOCK_DEV void st_tile_load(const void* kc, const void* vc, int kv_bf16, size_t kvs, int g,
                            int t0, int nt, int pos, StTile& tl) {
  const int t = threadIdx.x;
#pragma unroll
  for (int u = 0; u < ST_TILE_PER; u++) {
    const int e = t + u * ST_CTHREADS;  // float4 index in the tile
    const int j = e >> 5, c4 = e & 31, key = t0 + j;
    float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk;
    if (e < ST_TILE_F4 && j < nt && key != pos) {
      const size_t off = (size_t)key * kvs + (size_t)g * 128;
      if (kv_bf16) {
        const uint2 kw = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(kc) + off)[c4];
        const uint2 vw = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(vc) + off)[c4];
        const float2 k0 = bf16x2_widen(kw.x), k1 = bf16x2_widen(kw.y);
        const float2 v0 = bf16x2_widen(vw.x), v1 = bf16x2_widen(vw.y);
        kk = make_float4(k0.x, k0.y, k1.x, k1.y);
        vv = make_float4(v0.x, v0.y, v1.x, v1.y);
      } else {
        kk = __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(kc) + off) + c4);
        vv = __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(vc) + off) + c4);
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
FLOCK_DEV bool st_attention_item(const StArgs& a, const StLayer& L, int g, int s,
                                              int S, int pos, uint32_t tag,
                                              unsigned long long* tr, unsigned long long* det) {
  // the arguments this item needs, read once (see st_phase)
  const StCta c = st_cta(a);
  const int nH = a.nH, nKV = a.nKV, kv_bf16 = a.kv_bf16, neox = a.neox;
  const float eps = a.eps;
  const float* const inv_freq = a.inv_freq;
  const float2* const rope_cs = a.rope_cs;
  const int rope_rows = a.rope_rows;
  const uint64_t* const t_qkv = a.t_qkv;
  uint64_t* const t_part = a.t_part;
  uint64_t* const t_att = a.t_att;
  int* const err = a.err;
  void* const kc = L.kcache;
  void* const vc = L.vcache;
  const float* const qnorm = L.q_norm;
  const float* const knorm = L.k_norm;
  const int G = nH / nKV;
  auto mark = [&](int k) {
    if (det && threadIdx.x == 0) det[k] = globaltimer_ns();
  };
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float* xs = c.xs;
  const int n_keys = pos + 1;
  const int chunk = (n_keys + S - 1) / S;
  const int k0 = s * chunk, k1 = min(n_keys, k0 + chunk);
  const size_t kvs = (size_t)nKV * 128;
  bool ok = true;

  // the first tile's loads and the constant gains go out before the wait
  StTile tl;
  st_tile_load(kc, vc, kv_bf16, kvs, g, k0, min(ST_KT, k1 - k0), pos, tl);
  if (t < 32) {
    reinterpret_cast<float4*>(xs + SA_GQ)[t] = reinterpret_cast<const float4*>(qnorm)[t];
    reinterpret_cast<float4*>(xs + SA_GK)[t] = reinterpret_cast<const float4*>(knorm)[t];
  }
  if (t < 64) {
    float2* cs = reinterpret_cast<float2*>(xs + SA_CS);
    cs[t] = pos < rope_rows ? rope_cs[(size_t)pos * 64 + t] : rope_cs_at(pos, inv_freq[t]);
  }
  // q heads g*G .. g*G+G-1, k head g, v head g of the QKV output
  {
    const int nq = G * 128;
    const int qoff = g * G * 128, koff = nH * 128 + g * 128, voff = koff + nKV * 128;
    // word pairs: q [0, nq/2), k [nq/2, nq/2 + 64), v [.. + 64)
    const int npairs = nq / 2 + 128;
    for (int i = t; i < npairs; i += ST_CTHREADS) {
      const uint64_t* src;
      float* dst;
      if (i < nq / 2) {
        src = t_qkv + qoff + 2 * i;
        dst = xs + SA_QRAW + 2 * i;
      } else if (i < nq / 2 + 64) {
        src = t_qkv + koff + 2 * (i - nq / 2);
        dst = xs + SA_KRAW + 2 * (i - nq / 2);
      } else {
        src = t_qkv + voff + 2 * (i - nq / 2 - 64);
        dst = xs + SA_VRAW + 2 * (i - nq / 2 - 64);
      }
      ulonglong2 w = st_ld2(src);
      if (ok && !st_wait2(src, tag, w, err)) {
        atomicExch(err, ST_ERR_DATA);
        ok = false;
      }
      dst[0] = val_of(w.x);
      dst[1] = val_of(w.y);
    }
  }
  st_tile_store(tl, xs);
  if (st_any(!ok)) return false;
  if (tr && t == 0) tr[0] = globaltimer_ns();
  mark(0);
  // exact per-head RMSNorm + RoPE (k_qk_norm_rope_append's arithmetic)
  float* qv = xs + SA_QV;
  float* knew = xs + SA_KNEW;
  float* vnew = xs + SA_VNEW;
  if (warp < G)
    norm_rope_warp_cs(xs + SA_QRAW + warp * 128, xs + SA_GQ, eps,
                      reinterpret_cast<const float2*>(xs + SA_CS), neox,
                   qv + warp * 128, lane);
  else if (warp == G)
    norm_rope_warp_cs(xs + SA_KRAW, xs + SA_GK, eps, reinterpret_cast<const float2*>(xs + SA_CS),
                      neox, knew, lane);
  else if (warp == G + 1)
    for (int i = lane; i < 128; i += 32) vnew[i] = xs[SA_VRAW + i];
  st_bar();
  mark(1);
  const bool has_new = pos >= k0 && pos < k1;
  if (t < 128) {
    const size_t off = (size_t)pos * kvs + (size_t)g * 128 + t;
    if (kv_bf16) {
      // the cache keeps bf16: this step's scores use the rounded value too
      const uint16_t kb = bf16_bits(knew[t]), vb = bf16_bits(vnew[t]);
      knew[t] = __uint_as_float((uint32_t)kb << 16);
      vnew[t] = __uint_as_float((uint32_t)vb << 16);
      if (has_new) {
        static_cast<uint16_t*>(kc)[off] = kb;
        static_cast<uint16_t*>(vc)[off] = vb;
      }
    } else if (has_new) {
      static_cast<float*>(kc)[off] = knew[t];
      static_cast<float*>(vc)[off] = vnew[t];
    }
  }
  st_bar();
  mark(2);

  const float scale = __double2float_rn(1.0 / sqrt(128.0));
  float* kt = xs + SA_KT;
  float* vt = xs + SA_VT;
  // warp hq < G owns query head hq for the whole item: lane j scores key j
  // of a tile, the online softmax runs on warp shuffles, lane l accumulates
  // output dims 4l .. 4l + 3 -- no block barrier between a tile's scores,
  // softmax and P.V; m, l and o stay in registers
  float m = -INFINITY, lsum = 0.0f;
  float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4* q4 = reinterpret_cast<const float4*>(qv + (warp < G ? warp : 0) * 128);
  for (int t0 = k0; t0 < k1; t0 += ST_KT) {
    const int nt = min(ST_KT, k1 - t0);
    if (t0 != k0) {
      st_bar();  // the previous tile's readers are done
      st_tile_load(kc, vc, kv_bf16, kvs, g, t0, nt, pos, tl);
      st_tile_store(tl, xs);
      st_bar();  // the zero-filled row of key pos lands before it is overwritten below
    }
    if (pos >= t0 && pos < t0 + nt && t < 128) {
      kt[(pos - t0) * SA_KSTR + t] = knew[t];
      vt[(pos - t0) * 128 + t] = vnew[t];
    }
    st_bar();
    if (t0 == k0) mark(3);
    if (warp < G) {
      // rows 132 floats apart: each quarter-warp's 8 row reads hit distinct banks
      float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f, p3 = 0.0f;
      if (lane < nt) {
        const float4* kr = reinterpret_cast<const float4*>(kt + lane * SA_KSTR);
#pragma unroll 8
        for (int c4 = 0; c4 < 32; c4++) {
          const float4 kk = kr[c4], qq = q4[c4];
          p0 = fmaf(qq.x, kk.x, p0);
          p1 = fmaf(qq.y, kk.y, p1);
          p2 = fmaf(qq.z, kk.z, p2);
          p3 = fmaf(qq.w, kk.w, p3);
        }
      }
      const float v = lane < nt ? ((p0 + p1) + (p2 + p3)) * scale : -INFINITY;
      float mt = v;
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o2));
      const float m_new = fmaxf(m, mt);
      const float p = lane < nt ? expf(v - m_new) : 0.0f;
      float lt = p;
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o2);
      const float cr = expf(m - m_new);
      m = m_new;
      lsum = fmaf(lsum, cr, lt);
      o4 = make_float4(o4.x * cr, o4.y * cr, o4.z * cr, o4.w * cr);
      const float4* v4 = reinterpret_cast<const float4*>(vt) + lane;
      for (int j = 0; j < nt; j++) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const float4 vv = v4[j * 32];
        o4.x = fmaf(pj, vv.x, o4.x);
        o4.y = fmaf(pj, vv.y, o4.y);
        o4.z = fmaf(pj, vv.z, o4.z);
        o4.w = fmaf(pj, vv.w, o4.w);
      }
    }
  }
  mark(6);
  const int hq = warp;
  if (S == 1) {
    if (warp < G) {
      uint64_t* dst = t_att + (size_t)(g * G + hq) * 128 + 4 * lane;
      st_tag(dst, tag, o4.x / lsum);
      st_tag(dst + 1, tag, o4.y / lsum);
      st_tag(dst + 2, tag, o4.z / lsum);
      st_tag(dst + 3, tag, o4.w / lsum);
    }
    mark(7);
    return true;
  }
  if (s > 0) {  // this split's partial: unnormalised o, running max m, sum l
    if (warp < G) {
      uint64_t* pp = t_part + ((size_t)(g * G + hq) * ST_MAX_SPLITS + s) * ST_PSTRIDE;
      st_tag(pp + 4 * lane, tag, o4.x);
      st_tag(pp + 4 * lane + 1, tag, o4.y);
      st_tag(pp + 4 * lane + 2, tag, o4.z);
      st_tag(pp + 4 * lane + 3, tag, o4.w);
      if (lane == 0) {
        st_tag(pp + 128, tag, m);
        st_tag(pp + 129, tag, lsum);
      }
    }
    mark(7);
    return true;
  }
  // split 0 combines, warp hq for head hq: split weights w_s = e^(m_s - M)
  // (lane s holds splits s and s + 32), L = sum l_s w_s, then each lane sums
  // its 4 dims over the splits in order, 4 splits' loads in flight at a time
  if (warp < G) {
    const uint64_t* pp = t_part + (size_t)(g * G + hq) * ST_MAX_SPLITS * ST_PSTRIDE;
    float mv[2], lv[2];
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int sp = lane + 32 * u;
      mv[u] = -INFINITY;
      lv[u] = 0.0f;
      if (sp == 0) {
        mv[u] = m;
        lv[u] = lsum;
      } else if (sp < S) {
        ulonglong2 w = st_ld2(pp + (size_t)sp * ST_PSTRIDE + 128);
        if (ok && !st_wait2(pp + (size_t)sp * ST_PSTRIDE + 128, tag, w, err)) {
          atomicExch(err, ST_ERR_DATA);
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
    mark(7);
    const float ws0 = __shfl_sync(0xffffffffu, w0, 0);
    float4 O = make_float4(fmaf(o4.x, ws0, 0.0f), fmaf(o4.y, ws0, 0.0f), fmaf(o4.z, ws0, 0.0f),
                           fmaf(o4.w, ws0, 0.0f));
    for (int s0 = 1; s0 < S; s0 += 4) {
      ulonglong2 w[4][2];
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (s0 + u < S) {
          const uint64_t* q = pp + (size_t)(s0 + u) * ST_PSTRIDE + 4 * lane;
          w[u][0] = st_ld2(q);
          w[u][1] = st_ld2(q + 2);
        }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int sp = s0 + u;
        if (sp >= S) break;
        const uint64_t* q = pp + (size_t)sp * ST_PSTRIDE + 4 * lane;
        if (ok && !(st_wait2(q, tag, w[u][0], err) && st_wait2(q + 2, tag, w[u][1], err))) {
          atomicExch(err, ST_ERR_DATA);
          ok = false;
        }
        const float ws = __shfl_sync(0xffffffffu, sp >= 32 ? w1 : w0, sp & 31);
        O.x = fmaf(val_of(w[u][0].x), ws, O.x);
        O.y = fmaf(val_of(w[u][0].y), ws, O.y);
        O.z = fmaf(val_of(w[u][1].x), ws, O.z);
        O.w = fmaf(val_of(w[u][1].y), ws, O.w);
      }
    }
    uint64_t* dst = t_att + (size_t)(g * G + hq) * 128 + 4 * lane;
    st_tag(dst, tag, O.x / Lsum);
    st_tag(dst + 1, tag, O.y / Lsum);
    st_tag(dst + 2, tag, O.z / Lsum);
    st_tag(dst + 3, tag, O.w / Lsum);
  }
  mark(8);
  return ok;
}

// The producer warp: stream this CTA's pieces into the ring in order.
// The producer warp: lane s (< ring_slots) owns ring slot s and streams the
// CTA's pieces s, s + ring_slots, ... into it, each lane with its next
// descriptor already loaded.  One lane per slot lets the slots' drain waits
// and copy issues overlap; a single issuing thread paid its wake-up and
// issue latency once per piece (about 0.35 us), which capped a 16 KiB ring
// near 16 GB/s per SM against the 44 GB/s a full HBM stream needs.
FLOCK_DEV void st_producer(const StArgs& a) {
  const StCta c = st_cta(a);
  const int lane = threadIdx.x & 31;
  const StPiece* P = a.pieces + (size_t)blockIdx.x * a.max_pieces;
  const int np = a.n_pieces[blockIdx.x];
  const int ns = a.ring_slots;
  int* const err = a.err;
  const bool trace = a.trace != nullptr;
  unsigned long long wait_ns = 0;
  int issued = 0;
  int i = lane;
  if (lane < ns) {
    const int slot = lane;
    const int ahead = a.l2_rounds * ns;  // the L2 prefetch runs this many pieces ahead
    uint4 d0 = make_uint4(0, 0, 0, 0), d1 = d0, d2 = d0, f0 = d0, f1 = d0, f2 = d0;
    if (i < np) {
      const uint4* src = reinterpret_cast<const uint4*>(P + i);
      d0 = __ldg(src);
      d1 = __ldg(src + 1);
      d2 = __ldg(src + 2);
    }
    if (ahead > 0 && i + ahead < np) {
      const uint4* src = reinterpret_cast<const uint4*>(P + i + ahead);
      f0 = __ldg(src);
      f1 = __ldg(src + 1);
      f2 = __ldg(src + 2);
    }
    for (; i < np; i += ns) {
      const uint4 h0 = d0, h1 = d1, h2 = d2;
      if (i + ns < np) {  // the next descriptor of this slot, in flight during the wait
        const uint4* src = reinterpret_cast<const uint4*>(P + i + ns);
        d0 = __ldg(src);
        d1 = __ldg(src + 1);
        d2 = __ldg(src + 2);
      }
      if (ahead > 0 && i + ahead < np) {
        // weights do not depend on activations: stream the piece `ahead`
        // into L2 while the ring drains, so its ring copy later reads L2
        const uint32_t fn = f2.z >> 16;
        const uint32_t qsb = fn * f2.x, scb = fn * (f2.z & 0xFFFFu);
        const int nsub = ((f2.w & 0xFFFFu) & ST_PAIR) ? 2 : 1;
        if (fn != 0) {
          prefetch_l2(reinterpret_cast<const void*>(((uint64_t)f0.y << 32) | f0.x), qsb);
          prefetch_l2(reinterpret_cast<const void*>(((uint64_t)f1.y << 32) | f1.x), scb);
          if (nsub == 2) {
            prefetch_l2(reinterpret_cast<const void*>(((uint64_t)f0.w << 32) | f0.z), qsb);
            prefetch_l2(reinterpret_cast<const void*>(((uint64_t)f1.w << 32) | f1.z), scb);
          }
        }
        if (i + ns + ahead < np) {
          const uint4* src = reinterpret_cast<const uint4*>(P + i + ns + ahead);
          f0 = __ldg(src);
          f1 = __ldg(src + 1);
          f2 = __ldg(src + 2);
        }
      }
      const uint32_t round = (uint32_t)(i / ns);
      const uint64_t w0 = trace ? globaltimer_ns() : 0;
      if (round > 0 && !mbar_wait_poll(&c.empty[slot], (round - 1) & 1u, err)) {
        atomicExch(err, ST_ERR_RING);
        break;
      }
      if (w0) wait_ns += globaltimer_ns() - w0;
      uint4* h = reinterpret_cast<uint4*>(&c.hdr[slot]);
      h[0] = h0;
      h[1] = h1;
      h[2] = h2;
      // header words: d0 = qs[0..1], d1 = sc[0..1], d2 = {row_bytes, out_row,
      // sc_row | nrows << 16, flags | pad << 16}
      const uint32_t nrows = h2.z >> 16, flags = h2.w & 0xFFFFu;
      const uint32_t qsb = nrows * h2.x, scb = nrows * (h2.z & 0xFFFFu);
      const int nsub = (flags & ST_PAIR) ? 2 : 1;
      mbar_expect_tx(&c.full[slot], nrows ? nsub * (qsb + scb) : 0u);
      if (nrows) {
        uint8_t* dst = c.ring + (size_t)slot * ST_SLOT;
        bulk_g2s(dst, reinterpret_cast<const void*>(((uint64_t)h0.y << 32) | h0.x), qsb, &c.full[slot]);
        bulk_g2s(dst + qsb, reinterpret_cast<const void*>(((uint64_t)h1.y << 32) | h1.x), scb,
                 &c.full[slot]);
        if (nsub == 2) {
          dst += qsb + scb;
          bulk_g2s(dst, reinterpret_cast<const void*>(((uint64_t)h0.w << 32) | h0.z), qsb,
                   &c.full[slot]);
          bulk_g2s(dst + qsb, reinterpret_cast<const void*>(((uint64_t)h1.w << 32) | h1.z), scb,
                   &c.full[slot]);
        }
      }
      issued++;
    }
    c.flags[8 + slot] = i;  // the first piece of this slot not issued
    atomicAdd(&c.flags[0], issued);
  }
  if (trace && lane == 0) {
    unsigned long long* tr = a.trace + (size_t)blockIdx.x * st_trace_stride(a.n_layers);
    tr[6 + 10 * a.n_layers] = wait_ns;  // slot 0's lane
  }
}

// __grid_constant__: the phases read the arguments where the launch put them
// (a copy per thread would live in local memory).  Everything is inlined:
// with 224 KB of shared memory only ~30 KB of L1 is left, so local memory
// (spills, call frames) would cost an L2 round trip; the per-token scalars
// live in shared memory so the layer loop carries almost no registers.
// XH: hidden <= 1024, so the rows of the QKV, gate/up and head phases are one
// block per lane with x in registers (one instantiation per shape class
// keeps the kernel's code, and its instruction-cache footprint, smaller).
template <bool XH>
__global__ void __launch_bounds__(ST_THREADS, 1)
    k_decode_stream(const __grid_constant__ StArgs a) {
  int pi = 0;  // the compute threads' next piece
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    const StCta c = st_cta(a);
    if (threadIdx.x == 0) {
      for (int i = 0; i < a.ring_slots; i++) {
        mbar_init(&c.full[i], 1);
        mbar_init(&c.empty[i], ST_CWARPS);
      }
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      const int pos = a.ctl[0] + a.ctl[1];
      c.flags[0] = 0;
      c.flags[1] = 0;
      c.flags[2] = pos;
      c.flags[3] = (int)*a.seq;
      c.flags[4] = st_splits(pos + 1, a.splits_max);
      *c.wait_ns = 0;
      if (a.trace) {
        unsigned long long* tr = a.trace + (size_t)blockIdx.x * st_trace_stride(a.n_layers);
        tr[0] = globaltimer_ns();
        for (int i = 1; i < st_trace_stride(a.n_layers); i++)
          if (i < 6 + 10 * a.n_layers || i >= 8 + 10 * a.n_layers) tr[i] = 0;  // not the producer's
      }
    }
    if (threadIdx.x < ST_CWARPS) {
      c.am_v[threadIdx.x] = -FLT_MAX;
      c.am_i[threadIdx.x] = 0xFFFFFFFFu;
    }
  }
  __syncthreads();

  if (warp == ST_CWARPS) {
    st_producer(a);
  } else {
    auto stamp = [&](int i) {
      if (a.trace && threadIdx.x == 0)
        a.trace[(size_t)blockIdx.x * st_trace_stride(a.n_layers) + i] = globaltimer_ns();
    };
    const int t = threadIdx.x;
    // shared-memory regions, recomputed where used (st_cta is a few integer
    // ops on the arguments): keeping them live across the layer loop costs
    // registers the row folds need
#define C_ (st_cta(a))
    auto pdet = [&](int off, bool last) -> unsigned long long* {
      return (a.trace && last) ? a.trace + (size_t)blockIdx.x * st_trace_stride(a.n_layers) + 20 +
                                     10 * a.n_layers + off
                               : nullptr;
    };
    {
      // layer 0's input: the embedded token (k_embed's arithmetic), computed
      // by every CTA
      const int token = a.ids[0];
      for (int q = t; q < a.H / 4; q += ST_CTHREADS) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (token >= 0 && token < a.vocab) {
          const uint32_t w =
              *reinterpret_cast<const uint32_t*>(a.embd_qs + (size_t)token * a.H + 4 * q);
          const float sc = scale_f16(a.embd_sc[(size_t)token * a.embd_sc_stride + q / 8]);
          float q0, q1, q2, q3;
          dec_i8x4(w, q0, q1, q2, q3);
          v = make_float4(fmul(q0, sc), fmul(q1, sc), fmul(q2, sc), fmul(q3, sc));
        }
        reinterpret_cast<float4*>(C_.hs)[q] = v;
      }
    }
    stamp(1);
    // The token as a flat sequence of steps -- per layer QKV, attention,
    // o_proj, gate/up, down, then the head -- each code path compiled once:
    // acquire the step's input vector (poll its tagged words; RMSNorm into
    // the packed x when the step has a gain), then fold its rows.  Every
    // fallible step ends in st_any, so `ok` is uniform over the CTA.
    bool ok = true;
    const int L = a.n_layers;
    float* const hs = C_.hs;
    float* const xs = C_.xs;
    for (int st = 0; st < 5 * L + (a.head ? 1 : 0) && ok; st++) {
      const int l = st / 5, k = st - 5 * l;
      const bool head = l == L;
      const int kind = head ? ST_HEAD : k == 0 ? ST_QKV : k == 2 ? ST_O : k == 3 ? ST_GU
                                                                         : ST_DOWN;
      const uint32_t tag = ((uint32_t)C_.flags[3] << 8) | (uint32_t)(head ? L - 1 : l);
      const bool last = l == L - 1;
      if (!head && k == 1) {
        // ---- attention items of this CTA (at most one: items <= grid)
        const int S = C_.flags[4];
        for (int item = blockIdx.x; item < a.nKV * S; item += gridDim.x) {
          unsigned long long* tr =
              a.trace ? a.trace + (size_t)blockIdx.x * st_trace_stride(L) + 4 + 10 * l : nullptr;
          unsigned long long* det = (tr && last) ? tr - 4 - 10 * l + 8 + 10 * L : nullptr;
          ok = st_attention_item(a, a.layers[l], item / S, item % S, S, C_.flags[2], tag, tr, det);
          if (st_any(!ok)) ok = false;
          if (!ok) break;
        }
        stamp(5 + 10 * l);
        continue;
      }
      // ---- the step's input: h (QKV, gate/up, head: RMSNorm-ed) or the
      // attention output / act (o_proj, down: packed as they are)
      const float* gain = kind == ST_QKV ? a.layers[l].attn_norm
                          : kind == ST_GU ? a.layers[l].ffn_norm
                          : kind == ST_HEAD ? a.out_norm : nullptr;
      if (gain)
        for (int i = t; i < a.H; i += ST_CTHREADS) C_.gs[i] = __ldg(gain + i);
      if (kind != ST_QKV || l > 0) {
        const uint64_t* src = kind == ST_O ? a.t_att : kind == ST_GU ? a.t_ho
                              : kind == ST_DOWN ? a.t_act : a.t_hd;
        const int n = kind == ST_O ? a.nH * a.hd : kind == ST_DOWN ? a.F : a.H;
        // the QKV step reads the previous layer's h
        ok = st_poll_vec(src, n, kind == ST_QKV ? tag - 1 : tag, gain ? hs : xs, !gain, a.err);
      }
      if (st_any(!ok)) {
        ok = false;
        break;
      }
      const int sbase = head ? 2 + 10 * L : (kind == ST_QKV ? 2 : kind == ST_O ? 6 : kind == ST_GU
                                                                                ? 8 : 10) + 10 * l;
      stamp(sbase);
      if (gain) st_rmsnorm(hs, C_.gs, a.H, a.eps, xs, C_.red);
      // ---- its rows
      unsigned long long* pd =
          pdet(kind == ST_QKV ? 0 : kind == ST_GU ? 9 : 18, last && kind != ST_O && !head);
      const bool xr = XH && (kind == ST_QKV || kind == ST_GU || kind == ST_HEAD);
      const int np = xr ? st_phase<true>(a, pi, kind, tag, last, pd)
                        : st_phase<false>(a, pi, kind, tag, last, pd);
      ok = np >= 0;
      if (ok) pi = np;
      stamp(sbase + 1);
      if (st_any(!ok)) ok = false;
    }
    // CTA argmax over the warps' slots, then the last CTA reduces the grid's
    // (kernels/argmax.wgsl pass 1 / pass 2; lowest index on ties)
    st_bar();
    if (t == 0) {
      float bv = C_.am_v[0];
      uint32_t bi = C_.am_i[0];
      for (int w = 1; w < ST_CWARPS; w++)
        if (am_better(C_.am_v[w], C_.am_i[w], bv, bi)) {
          bv = C_.am_v[w];
          bi = C_.am_i[w];
        }
      a.am_val[blockIdx.x] = bv;
      a.am_idx[blockIdx.x] = bi;
      __threadfence();
      const uint32_t prev = atomicAdd(a.am_count, 1u);
      C_.flags[1] = prev == gridDim.x - 1;
    }
    st_bar();
    if (C_.flags[1]) {
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
        C_.am_v[warp] = bv;
        C_.am_i[warp] = bi;
      }
      st_bar();
      if (t == 0) {
        bv = C_.am_v[0];
        bi = C_.am_i[0];
        for (int w = 1; w < ST_CWARPS; w++)
          if (am_better(C_.am_v[w], C_.am_i[w], bv, bi)) {
            bv = C_.am_v[w];
            bi = C_.am_i[w];
          }
        const int pos = C_.flags[2];
        if (!*(volatile int*)a.err) {
          if (a.head) {  // else the head GEMV writes the id and the history slot
            a.ids[0] = (int32_t)bi;
            if (pos >= 0 && pos < a.hist_cap) a.hist[pos] = (int32_t)bi;
          }
          a.ctl[0] = pos;
          a.ctl[1] = 1;
        }
        // next launch's tags; 24 bits of sequence, never 0
        *a.seq = ((uint32_t)C_.flags[3] % 0xFFFFFEu) + 1u;
        *a.am_count = 0;
      }
    }
    stamp(4 + 10 * a.n_layers);
    if (a.trace && threadIdx.x == 0)
      a.trace[(size_t)blockIdx.x * st_trace_stride(a.n_layers) + 5 + 10 * a.n_layers] = *C_.wait_ns;
  }
#undef C_
  __syncthreads();
  // every bulk copy issued must land before the CTA exits: wait (bounded)
  // for the pieces issued but not consumed (only after an error; at most one
  // per slot beyond the consumers' position)
  if (threadIdx.x == 0) {
    const StCta c = st_cta(a);
    for (int i = pi; i < pi + a.ring_slots; i++) {
      const int slot = i % a.ring_slots;
      if (i < c.flags[8 + slot])
        mbar_wait(&c.full[slot], (uint32_t)(i / a.ring_slots) & 1u, a.err, false);
    }
    if (a.trace)
      a.trace[(size_t)blockIdx.x * st_trace_stride(a.n_layers) + 7 + 10 * a.n_layers] =
          (unsigned long long)c.flags[0];
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
  return xb + (size_t)H * 4 + (size_t)hf * 4 + 136 * 4 + ST_CWARPS * 32 * 4 + ST_CWARPS * 8 + 8 +
         (8 + 32) * 4;
}
inline size_t st_smem_bytes(int slots, size_t fixed) {
  return (size_t)slots * (ST_SLOT + sizeof(StPiece) + 16) + fixed;
}

}  // namespace flock
