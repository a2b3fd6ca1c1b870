// Persistent decode kernel: one cooperative launch per generated token.
//
// Same arithmetic as the per-op kernels (k_embed, k_gemv, k_attn_decode_fast)
// -- it calls the same device functions in the same order, so its logits and
// ids are bit-identical to the multi-kernel path -- but laid out for batch-1
// latency on B200:
//
//  * one CTA per SM: 8 consumer warps compute, 1 producer warp streams the
//    CTA's weight rows for the coming phases into a ring of shared-memory
//    stages with cp.async.bulk (TMA bulk copies completing on mbarriers).
//    Weights do not depend on activations, so the producer runs ahead across
//    the grid barriers and the next phase's rows are usually resident before
//    the barrier releases;
//  * phases per layer: QKV (attn_norm fused) | attention (split-K, q/k norm +
//    RoPE + KV append fused) | o_proj + residual | gate/up (ffn_norm fused) +
//    SwiGLU | down + residual, separated by grid barriers (release-add /
//    acquire-poll on one counter); layer 0's embedding is computed by every
//    CTA redundantly so it needs no barrier;
//  * the LM head streams 1/148 of the 151936 rows per CTA through the ring,
//    with the argmax reduced per CTA and finished by the last CTA to arrive,
//    which also writes the chosen id, its history slot and the position.
//
// Every wait is bounded: on a timeout the kernel sets *err, skips the rest
// of the work, drains its own bulk copies (bounded) and returns; the host
// reports the error.  No multicast loads are used.
#pragma once
#include "attn_fast.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "mbar.cuh"

namespace flock {

struct MkLayer {
  const uint8_t* qs[7];   // q, k, v, o, gate, up, down
  const uint16_t* sc[7];
  int sc_stride[7];
  const float* attn_norm;
  const float* q_norm;
  const float* k_norm;
  const float* ffn_norm;
  float* kcache;
  float* vcache;
};

struct MkArgs {
  const MkLayer* layers;
  int n_layers;
  int H, nH, nKV, hd, F, vocab;
  float eps;
  int neox;
  const float* inv_freq;
  const uint8_t* embd_qs;
  const uint16_t* embd_sc;
  int embd_sc_stride;
  const uint8_t* head_qs;
  const uint16_t* head_sc;
  int head_sc_stride;
  const float* out_norm;
  float* h;       // [H]
  float* q;       // [nH*hd]
  float* k;       // [nKV*hd]
  float* v;       // [nKV*hd]
  float* attn;    // [nH*hd]
  float* act;     // [F]
  float* logits;  // [vocab]
  int32_t* ids;   // ids[0]: input token in, chosen token out
  int32_t* hist;
  int hist_cap;
  float* attn_part;
  uint32_t* attn_count;
  int splits;
  float* am_val;
  uint32_t* am_idx;
  uint32_t* am_count;
  float* am_best_val;
  int* ctl;        // {pos of the previous step's first token, n_last}
  unsigned* bar;   // grid barrier counter, zero at launch
  int* err;        // set non-zero on a timed-out wait
  int stage_bytes; // bytes per ring stage
  int n_stages;
  // optional phase trace: per CTA, mk_trace_stride(n_layers) entries of
  // global-timer nanoseconds -- stamps (start, embedded, then per layer and
  // phase: computed, released; head computed, done), then the time warp 0
  // waited for weights in the QKV, o_proj, gate/up, down and head phases
  // (summed over layers) and the time the producer waited for a free stage;
  // nullptr when off
  unsigned long long* trace;
};

__host__ __device__ inline int mk_trace_stride(int n_layers) { return 10 + 10 * n_layers; }

constexpr int MK_CONSUMERS = 8;                   // consumer warps
constexpr int MK_THREADS = (MK_CONSUMERS + 1) * 32;
constexpr int MK_MAX_STAGES = 8;
FLOCK_DEV unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
FLOCK_DEV void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// named barrier over the consumer warps only (the producer never joins)
FLOCK_DEV void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(MK_CONSUMERS * 32) : "memory");
}

// ----------------------------------------------------------- the schedule
//
// The token's weight stream is a fixed sequence of chunks that producer and
// consumers walk identically.  A phase p (per layer: 0 QKV, 1 attention,
// 2 o_proj, 3 gate/up, 4 down; then 5 = head) gives this CTA a contiguous
// range of its row groups; the range is cut into chunks that fit one stage
// and never cross a tensor (segment) boundary.

enum { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_HEAD = 5 };

struct Chunk {
  int seg;     // tensor within the phase (QKV: 0 q, 1 k, 2 v; GU: 0 = gate+up pairs)
  int row0;    // first row within that tensor
  int rows;    // rows (GU: pairs)
  int K;       // columns
  uint32_t bytes;
};

struct PhaseGeo {
  int K;             // columns
  int units;         // row groups over the whole phase (GU: pairs)
  int nseg;          // QKV 3, others 1
  int seg_rows[3];   // rows per segment (QKV)
  int unit_bytes;    // shared-memory bytes one unit takes (qs + padded scales)
};

FLOCK_DEV PhaseGeo phase_geo(const MkArgs& a, int p) {
  PhaseGeo g{};
  const int qw = a.nH * a.hd, kvw = a.nKV * a.hd;
  auto scb = [](int K) { return ((K / 32 + 7) / 8 * 8) * 2; };
  if (p == PH_QKV) {
    g.K = a.H; g.nseg = 3; g.seg_rows[0] = qw; g.seg_rows[1] = kvw; g.seg_rows[2] = kvw;
    g.units = qw + 2 * kvw; g.unit_bytes = g.K + scb(g.K);
  } else if (p == PH_O) {
    g.K = qw; g.nseg = 1; g.seg_rows[0] = a.H; g.units = a.H; g.unit_bytes = g.K + scb(g.K);
  } else if (p == PH_GU) {
    g.K = a.H; g.nseg = 1; g.seg_rows[0] = a.F; g.units = a.F; g.unit_bytes = 2 * (g.K + scb(g.K));
  } else if (p == PH_DOWN) {
    g.K = a.F; g.nseg = 1; g.seg_rows[0] = a.H; g.units = a.H; g.unit_bytes = g.K + scb(g.K);
  } else if (p == PH_HEAD) {
    g.K = a.H; g.nseg = 1; g.seg_rows[0] = a.vocab; g.units = a.vocab; g.unit_bytes = g.K + scb(g.K);
  }
  return g;
}

// This CTA's unit range of a phase: an even split, remainder first.
FLOCK_DEV void cta_range(int units, int& u0, int& u1) {
  const int n = gridDim.x, c = blockIdx.x;
  const int base = units / n, extra = units % n;
  u0 = c * base + min(c, extra);
  u1 = u0 + base + (c < extra ? 1 : 0);
}

// Chunks of this CTA for phase p; `emit(Chunk)` is called in order.
template <typename F>
FLOCK_DEV void for_each_chunk(const MkArgs& a, int p, F&& emit) {
  if (p == PH_ATT) return;
  const PhaseGeo g = phase_geo(a, p);
  int u0, u1;
  cta_range(g.units, u0, u1);
  const int per = max(1, a.stage_bytes / g.unit_bytes);
  int segbase = 0;
  for (int s = 0; s < g.nseg; s++) {
    const int lo = max(u0, segbase), hi = min(u1, segbase + g.seg_rows[s]);
    for (int r = lo; r < hi; r += per) {
      Chunk c;
      c.seg = s;
      c.row0 = r - segbase;
      c.rows = min(per, hi - r);
      c.K = g.K;
      c.bytes = (uint32_t)(c.rows * g.unit_bytes);
      emit(c);
    }
    segbase += g.seg_rows[s];
  }
}

// ---------------------------------------------------------------- producer
FLOCK_DEV void chunk_sources(const MkArgs& a, int layer, int p, const Chunk& c,
                             const uint8_t** qs, const uint16_t** sc, int* scs, int* nsrc) {
  if (p == PH_HEAD) {
    qs[0] = a.head_qs; sc[0] = a.head_sc; scs[0] = a.head_sc_stride; *nsrc = 1;
    return;
  }
  const MkLayer& L = a.layers[layer];
  int t0 = 0;
  if (p == PH_QKV) t0 = c.seg;        // q, k or v
  else if (p == PH_O) t0 = 3;
  else if (p == PH_GU) t0 = 4;        // gate and up
  else if (p == PH_DOWN) t0 = 6;
  qs[0] = L.qs[t0]; sc[0] = L.sc[t0]; scs[0] = L.sc_stride[t0]; *nsrc = 1;
  if (p == PH_GU) {
    qs[1] = L.qs[5]; sc[1] = L.sc[5]; scs[1] = L.sc_stride[5]; *nsrc = 2;
  }
}

// Stage layout of a chunk: [qs of src 0][qs of src 1][scales of src 0][scales of src 1]
FLOCK_DEV void issue_chunk(const MkArgs& a, int layer, int p, const Chunk& c, uint8_t* stage,
                           uint64_t* full) {
  const uint8_t* qs[2];
  const uint16_t* sc[2];
  int scs[2], nsrc;
  chunk_sources(a, layer, p, c, qs, sc, scs, &nsrc);
  mbar_expect_tx(full, c.bytes);
  const uint32_t qbytes = (uint32_t)c.rows * c.K;
  for (int i = 0; i < nsrc; i++)
    bulk_g2s(stage + i * qbytes, qs[i] + (size_t)c.row0 * c.K, qbytes, full);
  uint8_t* scdst = stage + nsrc * qbytes;
  for (int i = 0; i < nsrc; i++) {
    const uint32_t sb = (uint32_t)c.rows * scs[i] * 2;
    bulk_g2s(scdst + i * sb, sc[i] + (size_t)c.row0 * scs[i], sb, full);
  }
}

// ---------------------------------------------------------------- consumer
// One Q8_0 block of a row held in shared memory.
FLOCK_DEV void load_block_smem(BlockW<QT_Q8>& bw, const uint8_t* row_qs, const uint16_t* row_sc,
                               int b) {
  const uint4* p = reinterpret_cast<const uint4*>(row_qs + (size_t)b * 32);
  bw.w0 = p[0];
  bw.w1 = p[1];
  bw.s = row_sc[b];
}

// Grid barrier over all CTAs (consumer warps only).  Bounded; on timeout or
// a prior error anywhere it returns false and the caller stops working.
FLOCK_DEV bool grid_barrier(const MkArgs& a, unsigned& epoch) {
  consumers_sync();
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    epoch += 1;
    const unsigned target = epoch * gridDim.x;
    red_release_add(a.bar, 1u);
    int ok = 1;
    uint64_t t0 = 0;
    for (uint32_t i = 0; ld_acquire_u32(a.bar) < target; i++) {
      if ((i & 31) != 31) continue;
      if (*(volatile int*)a.err) { ok = 0; break; }
      const uint64_t now = globaltimer_ns();
      if (!t0) t0 = now;
      if (now - t0 > WAIT_NS || i >= WAIT_MAX_POLLS) {
        atomicExch(a.err, 2);
        ok = 0;
        break;
      }
    }
    s_ok = ok;
  }
  consumers_sync();
  return s_ok != 0;
}


struct ConsumerSync {
  FLOCK_DEV void operator()() const { consumers_sync(); }
};

// x lives in shared memory in gemv.cuh's packed-pair layout (xperm<QT_Q8>),
// folded with fold_block_packed; the norm gains are staged the same way.

// x for a GEMV phase: one round trip of 128-bit loads into the packed shared
// layout, then each lane's block 0 of x into registers (xp).  With `gain`,
// RMSNorm is fused in the exact ops_ref.ts:20 order (WG = 128: partial t
// folds elements t, t+128, ...; partials t and t+64, then t+32, then the
// shuffle tree): every warp computes the scale itself from shared memory, so
// one consumer barrier suffices when a row's x fits lane-resident blocks
// (K <= 1024); larger K also rescales the shared copy.  `src` is global
// memory written before the last grid barrier, or shared memory.
FLOCK_DEV void mk_stage(const float* src, bool src_shared, int K, const float* gain, float eps,
                        float* xs, float* gs, uint64_t (&xp)[16]) {
  const int t = threadIdx.x, lane = t & 31;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  const float4* g4 = reinterpret_cast<const float4*>(gain);
  for (int i = t; i < K / 8; i += MK_CONSUMERS * 32) {
    const float4 a = src_shared ? s4[2 * i] : __ldcg(s4 + 2 * i);
    const float4 b = src_shared ? s4[2 * i + 1] : __ldcg(s4 + 2 * i + 1);
    float4* d = reinterpret_cast<float4*>(xs + (i >> 2) * XPAD + (i & 3) * 8);
    d[0] = make_float4(a.x, b.x, a.y, b.y);
    d[1] = make_float4(a.z, b.z, a.w, b.w);
    if (gain) {
      const float4 ga = __ldg(g4 + 2 * i), gb = __ldg(g4 + 2 * i + 1);
      float4* e = reinterpret_cast<float4*>(gs + (i >> 2) * XPAD + (i & 3) * 8);
      e[0] = make_float4(ga.x, gb.x, ga.y, gb.y);
      e[1] = make_float4(ga.z, gb.z, ga.w, gb.w);
    }
  }
  consumers_sync();
  const int nb = K / 32;
  if (!gain) {
    if (lane < nb) load_pairs(xs, lane, xp);
    return;
  }
  float p[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int q = 0; q < 4; q++)
    for (int i = lane + 32 * q; i < K; i += 128) {
      const float v = xs[xperm<QT_Q8>(i)];
      p[q] = ffma(v, v, p[q]);
    }
  float v = fadd(fadd(p[0], p[2]), fadd(p[1], p[3]));
  v = warp_tree_sum(v);
  v = __shfl_sync(0xffffffffu, v, 0);
  const float scale = rsqrt_f64r(fadd(fdiv(v, (float)K), eps));
  if (nb <= 32) {
    if (lane < nb) {
      const float4* x4 = reinterpret_cast<const float4*>(xs + lane * XPAD);
      const float4* w4 = reinterpret_cast<const float4*>(gs + lane * XPAD);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float4 x = x4[j], g = w4[j];
        xp[2 * j] = pack2(fmul(fmul(x.x, scale), g.x), fmul(fmul(x.y, scale), g.y));
        xp[2 * j + 1] = pack2(fmul(fmul(x.z, scale), g.z), fmul(fmul(x.w, scale), g.w));
      }
    }
    return;
  }
  consumers_sync();  // every warp has read the unscaled copy
  for (int i = t; i < K; i += MK_CONSUMERS * 32) {
    const int o = xperm<QT_Q8>(i);
    xs[o] = fmul(fmul(xs[o], scale), gs[o]);
  }
  consumers_sync();
  load_pairs(xs, lane, xp);
}

// x for o_proj: the attention output, combined here from the split partials
// the attention phase left (attn_combine_warp, one warp per query head --
// the same arithmetic as the kernel graph's last-split combine).
FLOCK_DEV void mk_stage_attn(const MkArgs& a, int pos, float* xs, uint64_t (&xp)[16]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int splits = attn_splits_for(pos + 1, a.splits);
  for (int h = warp; h < a.nH; h += MK_CONSUMERS)
    attn_combine_warp(a.attn_part + (size_t)h * a.splits * (a.hd + 2), splits, a.hd, lane,
                      [&](int i, float v) { xs[xperm<QT_Q8>(h * a.hd + i)] = v; });
  consumers_sync();
  if (lane < a.nH * a.hd / 32) load_pairs(xs, lane, xp);
}

// R rows held in shared memory against the staged x, interleaved so their
// dependency chains overlap: the reference's coop(64) order per row (lane
// plays logical lanes lane and lane+32; block 0 of x from registers, the rest
// from the packed shared copy), then the 64-lane tree.  Lane 0 gets y[r].
template <int R>
FLOCK_DEV void mk_rows_dot(const uint8_t* const* rq, const uint16_t* const* rs, int nb,
                           const uint64_t (&xp)[16], const float* xs, int lane, float* y) {
  float accA[R], accB[R];
#pragma unroll
  for (int r = 0; r < R; r++) accA[r] = accB[r] = 0.0f;
  const int M = (nb + 31) / 32;
  for (int m = 0; m < M; m++) {
    const int b = lane + 32 * m;
    if (b >= nb) break;
    BlockW<QT_Q8> bw[R];
#pragma unroll
    for (int r = 0; r < R; r++) load_block_smem(bw[r], rq[r], rs[r], b);
    if (m == 0) {
#pragma unroll
      for (int r = 0; r < R; r++) accA[r] = fold_block_packed<QT_Q8>(bw[r], xp, accA[r]);
    } else {
      uint64_t xb[16];
      load_pairs(xs, b, xb);
      if (m & 1) {
#pragma unroll
        for (int r = 0; r < R; r++) accB[r] = fold_block_packed<QT_Q8>(bw[r], xb, accB[r]);
      } else {
#pragma unroll
        for (int r = 0; r < R; r++) accA[r] = fold_block_packed<QT_Q8>(bw[r], xb, accA[r]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) y[r] = fadd(accA[r], accB[r]);
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) {
#pragma unroll
    for (int r = 0; r < R; r++) y[r] = fadd(y[r], __shfl_down_sync(0xffffffffu, y[r], s));
  }
}

struct MkShared {
  float* xs;      // padded x
  float* gs;      // gain staging
  float* raw;     // [H] embedded row (layer 0)
  float* wv;      // [MK_CONSUMERS] argmax values
  uint32_t* wi;   // [MK_CONSUMERS] argmax indices
  float* att;     // AF_END floats for the attention phase (aliases the above)
};

// A warp's group of units (rows; gate/up: row pairs) within a chunk.  The
// group grows with the chunk (1, 2 or 4 units) so small chunks still spread
// over all consumer warps and large ones overlap several rows' chains.
template <int P, int U>
FLOCK_DEV void mk_group(const MkArgs& a, const Chunk& c, const uint8_t* q0, const uint8_t* q1,
                        const uint16_t* s0, const uint16_t* s1, int scs, int u0,
                        const uint64_t (&xp)[16], const float* xs, int lane, float& best_v,
                        uint32_t& best_i) {
  constexpr int R = P == PH_GU ? 2 * U : U;  // row dots
  const uint8_t* rq[R];
  const uint16_t* rs[R];
#pragma unroll
  for (int r = 0; r < U; r++) {
    const int u = min(u0 + r, c.rows - 1);  // a short group repeats its last unit
    rq[r] = q0 + (size_t)u * c.K;
    rs[r] = s0 + (size_t)u * scs;
    if (P == PH_GU) {
      rq[U + r] = q1 + (size_t)u * c.K;
      rs[U + r] = s1 + (size_t)u * scs;
    }
  }
  float y[R];
  mk_rows_dot<R>(rq, rs, c.K / 32, xp, xs, lane, y);
  if (lane != 0) return;
#pragma unroll
  for (int r = 0; r < U; r++) {
    if (u0 + r >= c.rows) break;
    const int row = c.row0 + u0 + r;
    if (P == PH_GU) {
      // ops_ref.ts:103 swigluRef: fr(fr(g / fr(1 + fr(exp(-g)))) * up)
      const float e = exp_f64r(-y[r]);
      a.act[row] = fmul(fdiv(y[r], fadd(1.0f, e)), y[U + r]);
    } else if (P == PH_QKV) {
      float* dst = c.seg == 0 ? a.q : (c.seg == 1 ? a.k : a.v);
      dst[row] = y[r];
    } else if (P == PH_O || P == PH_DOWN) {
      a.h[row] = fadd(__ldcg(a.h + row), y[r]);
    } else if (P == PH_HEAD) {
      a.logits[row] = y[r];
      if (am_better(y[r], (uint32_t)row, best_v, best_i)) {
        best_v = y[r];
        best_i = (uint32_t)row;
      }
    }
  }
}

// A GEMV phase over this CTA's chunks.  A weight wait that gives up sets *err.
template <int P>
FLOCK_DEV void mk_gemv_phase(const MkArgs& a, uint8_t* ring, uint64_t* full, uint64_t* empty,
                             int& cidx, const float* xs, const uint64_t (&xp)[16], float& best_v,
                             uint32_t& best_i, unsigned long long* wait_acc) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int UMAX = P == PH_GU ? 2 : 4;
  unsigned long long waited = 0;
  for_each_chunk(a, P, [&](const Chunk& c) {
    const int st = cidx % a.n_stages;
    const unsigned long long w0 = wait_acc ? globaltimer_ns() : 0;
    if (!mbar_wait(&full[st], (uint32_t)((cidx / a.n_stages) & 1), a.err)) atomicCAS(a.err, 0, 1);
    if (wait_acc) waited += globaltimer_ns() - w0;
    const uint8_t* stage = ring + (size_t)st * a.stage_bytes;
    const int scs = (c.K / 32 + 7) / 8 * 8;
    const int nsrc = P == PH_GU ? 2 : 1;
    const uint32_t qbytes = (uint32_t)c.rows * c.K;
    const uint8_t* q0 = stage;
    const uint8_t* q1 = stage + qbytes;
    const uint16_t* s0 = reinterpret_cast<const uint16_t*>(stage + nsrc * qbytes);
    const uint16_t* s1 = s0 + (size_t)c.rows * scs;
    int U = (c.rows + MK_CONSUMERS - 1) / MK_CONSUMERS;
    U = U > 2 ? UMAX : U;
    for (int u0 = warp * U; u0 < c.rows; u0 += MK_CONSUMERS * U) {
      if (U == 1)
        mk_group<P, 1>(a, c, q0, q1, s0, s1, scs, u0, xp, xs, lane, best_v, best_i);
      else if (U == 2)
        mk_group<P, 2>(a, c, q0, q1, s0, s1, scs, u0, xp, xs, lane, best_v, best_i);
      else
        mk_group<P, UMAX>(a, c, q0, q1, s0, s1, scs, u0, xp, xs, lane, best_v, best_i);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    cidx++;
  });
  if (wait_acc) *wait_acc += waited;
}

// The per-token kernel.  grid = one CTA per SM (cooperative), block =
// MK_THREADS, dynamic smem = ring + barriers + the x/attention region.
static __global__ void __launch_bounds__(MK_THREADS, 1) k_decode_mk(const MkArgs a) {
  extern __shared__ __align__(128) uint8_t mk_smem[];
  uint8_t* ring = mk_smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)a.n_stages * a.stage_bytes);
  uint64_t* empty = full + MK_MAX_STAGES;
  float* xregion = reinterpret_cast<float*>(empty + MK_MAX_STAGES);
  const int kmax = max(a.H, max(a.nH * a.hd, a.F));
  MkShared sm;
  sm.xs = xregion;
  sm.gs = sm.xs + kmax / 32 * XPAD;
  sm.raw = sm.gs + a.H / 32 * XPAD;
  sm.wv = sm.raw + a.H;
  sm.wi = reinterpret_cast<uint32_t*>(sm.wv + MK_CONSUMERS);
  sm.att = xregion;
  __shared__ bool att_last;
  __shared__ int s_issued[MK_MAX_STAGES];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.n_stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], MK_CONSUMERS);
      s_issued[s] = -1;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  unsigned long long* tr =
      a.trace ? a.trace + (size_t)blockIdx.x * mk_trace_stride(a.n_layers) : nullptr;
  auto stamp = [&](int i) {
    if (tr && threadIdx.x == 0) tr[i] = globaltimer_ns();
  };
  stamp(0);
  // weight-wait accumulators (thread 0) and the producer's stage wait
  unsigned long long* wacc = tr && threadIdx.x == 0 ? tr + 4 + 10 * a.n_layers : nullptr;
  if (wacc)
    for (int i = 0; i < 5; i++) wacc[i] = 0;
  const int pos = a.ctl[0] + a.ctl[1];  // this token's position
  const int token = a.ids[0];

  if (warp == MK_CONSUMERS) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int cidx = 0;
      bool stop = false;
      unsigned long long waited = 0;
      auto produce = [&](int layer, int p) {
        for_each_chunk(a, p, [&](const Chunk& c) {
          if (stop) return;
          const int st = cidx % a.n_stages;
          const unsigned long long w0 = tr ? globaltimer_ns() : 0;
          if (cidx >= a.n_stages &&
              !mbar_wait(&empty[st], (uint32_t)(((cidx / a.n_stages) - 1) & 1), a.err)) {
            stop = true;
            return;
          }
          if (tr) waited += globaltimer_ns() - w0;
          if (*(volatile int*)a.err) {
            stop = true;
            return;
          }
          issue_chunk(a, layer, p, c, ring + (size_t)st * a.stage_bytes, &full[st]);
          s_issued[st] = cidx;
          cidx++;
        });
      };
      for (int l = 0; l < a.n_layers && !stop; l++) {
        produce(l, PH_QKV);
        produce(l, PH_O);
        produce(l, PH_GU);
        produce(l, PH_DOWN);
      }
      if (!stop) produce(0, PH_HEAD);
      if (tr) tr[9 + 10 * a.n_layers] = waited;
    }
  } else {
    // ------------------------------------------------------------ consumers
    int cidx = 0;
    unsigned epoch = 0;
    float best_v = -FLT_MAX;
    uint32_t best_i = 0xFFFFFFFFu;
    // layer 0's input: every CTA embeds the token itself (k_embed's
    // arithmetic); CTA 0 also publishes it as the residual stream h.
    if (token >= 0 && token < a.vocab) {
      for (int g = threadIdx.x; g < a.H / 4; g += MK_CONSUMERS * 32) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(a.embd_qs + (size_t)token * a.H + 4 * g);
        const float sc = scale_f16(a.embd_sc[(size_t)token * a.embd_sc_stride + g / 8]);
        float q0, q1, q2, q3;
        dec_i8x4(w, q0, q1, q2, q3);
        reinterpret_cast<float4*>(sm.raw)[g] = make_float4(fmul(q0, sc), fmul(q1, sc), fmul(q2, sc), fmul(q3, sc));
      }
    } else {
      for (int g = threadIdx.x; g < a.H / 4; g += MK_CONSUMERS * 32)
        reinterpret_cast<float4*>(sm.raw)[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    consumers_sync();
    if (blockIdx.x == 0)
      for (int i = threadIdx.x; i < a.H; i += MK_CONSUMERS * 32) a.h[i] = sm.raw[i];
    stamp(1);

    AttnFastArgs aa = {};
    aa.q = a.q;
    aa.k = a.k;
    aa.v = a.v;
    aa.inv_freq = a.inv_freq;
    aa.out = a.attn;
    aa.part = a.attn_part;
    aa.count = a.attn_count;
    aa.n_heads = a.nH;
    aa.n_kv_heads = a.nKV;
    aa.head_dim = a.hd;
    aa.splits = a.splits;
    aa.eps = a.eps;
    aa.neox = a.neox;
    aa.combine = 0;  // the o_proj staging combines the partials
    uint64_t xr0[16];

    bool ok = true;
    for (int l = 0; l < a.n_layers && ok; l++) {
      const MkLayer& L = a.layers[l];
      // QKV (attn_norm fused)
      mk_stage(l == 0 ? sm.raw : a.h, l == 0, a.H, L.attn_norm, a.eps, sm.xs, sm.gs, xr0);
      mk_gemv_phase<PH_QKV>(a, ring, full, empty, cidx, sm.xs, xr0, best_v, best_i,
                              wacc ? wacc + 0 : nullptr);
      stamp(2 + l * 10 + 0);
      if (!(ok = grid_barrier(a, epoch))) break;
      stamp(2 + l * 10 + 1);
      // attention (q/k norm + RoPE + KV append fused)
      aa.q_norm = L.q_norm;
      aa.k_norm = L.k_norm;
      aa.kcache = L.kcache;
      aa.vcache = L.vcache;
      if ((int)blockIdx.x < a.nKV * a.splits)
        attn_fast_item(aa, blockIdx.x / a.splits, blockIdx.x % a.splits, pos, sm.att, &att_last,
                       ConsumerSync{});
      stamp(2 + l * 10 + 2);
      if (!(ok = grid_barrier(a, epoch))) break;
      stamp(2 + l * 10 + 3);
      // o_proj + residual
      mk_stage_attn(a, pos, sm.xs, xr0);
      mk_gemv_phase<PH_O>(a, ring, full, empty, cidx, sm.xs, xr0, best_v, best_i,
                              wacc ? wacc + 1 : nullptr);
      stamp(2 + l * 10 + 4);
      if (!(ok = grid_barrier(a, epoch))) break;
      stamp(2 + l * 10 + 5);
      // gate/up + SwiGLU (ffn_norm fused)
      mk_stage(a.h, false, a.H, L.ffn_norm, a.eps, sm.xs, sm.gs, xr0);
      mk_gemv_phase<PH_GU>(a, ring, full, empty, cidx, sm.xs, xr0, best_v, best_i,
                              wacc ? wacc + 2 : nullptr);
      stamp(2 + l * 10 + 6);
      if (!(ok = grid_barrier(a, epoch))) break;
      stamp(2 + l * 10 + 7);
      // down + residual
      mk_stage(a.act, false, a.F, nullptr, a.eps, sm.xs, sm.gs, xr0);
      mk_gemv_phase<PH_DOWN>(a, ring, full, empty, cidx, sm.xs, xr0, best_v, best_i,
                              wacc ? wacc + 3 : nullptr);
      stamp(2 + l * 10 + 8);
      ok = grid_barrier(a, epoch);
      stamp(2 + l * 10 + 9);
    }
    if (ok) {
    // output_norm + head + argmax
    mk_stage(a.h, false, a.H, a.out_norm, a.eps, sm.xs, sm.gs, xr0);
    mk_gemv_phase<PH_HEAD>(a, ring, full, empty, cidx, sm.xs, xr0, best_v, best_i,
                              wacc ? wacc + 4 : nullptr);
    stamp(2 + a.n_layers * 10);
    if (lane == 0) {
      sm.wv[warp] = best_v;
      sm.wi[warp] = best_i;
    }
    consumers_sync();
    __shared__ bool last;
    if (threadIdx.x == 0) {
      float bv = sm.wv[0];
      uint32_t bi = sm.wi[0];
      for (int w = 1; w < MK_CONSUMERS; w++)
        if (am_better(sm.wv[w], sm.wi[w], bv, bi)) {
          bv = sm.wv[w];
          bi = sm.wi[w];
        }
      a.am_val[blockIdx.x] = bv;
      a.am_idx[blockIdx.x] = bi;
      __threadfence();
      last = atomicAdd(a.am_count, 1u) == gridDim.x - 1;
    }
    consumers_sync();
    if (last && warp == 0) {
      // the CTA partials, one per lane at a time, then the shuffle tree
      __threadfence();
      float bv = -FLT_MAX;
      uint32_t bi = 0xFFFFFFFFu;
      for (int i = lane; i < (int)gridDim.x; i += 32) {
        const float v = __ldcg(a.am_val + i);
        const uint32_t ix = __ldcg(a.am_idx + i);
        if (am_better(v, ix, bv, bi)) {
          bv = v;
          bi = ix;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_down_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, o);
        if (am_better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        *a.am_best_val = bv;
        a.ids[0] = (int32_t)bi;
        if (pos >= 0 && pos < a.hist_cap) a.hist[pos] = (int32_t)bi;
        a.ctl[0] = pos;
        a.ctl[1] = 1;
        *a.am_count = 0;
      }
    }
    stamp(3 + a.n_layers * 10);
    }  // ok
  }
  __syncthreads();
  // Drain: never leave a bulk copy in flight into this CTA's shared memory.
  if (threadIdx.x == 0 && *(volatile int*)a.err) {
    for (int s = 0; s < a.n_stages; s++)
      if (s_issued[s] >= 0)
        mbar_wait(&full[s], (uint32_t)((s_issued[s] / a.n_stages) & 1), a.err, false);
  }
}

// Dynamic shared memory of a k_decode_mk launch.
inline size_t mk_smem_bytes(int stage_bytes, int n_stages, int H, int qw, int F) {
  const int kmax = H > qw ? (H > F ? H : F) : (qw > F ? qw : F);
  const size_t xfloats = (size_t)kmax / 32 * XPAD + (size_t)H / 32 * XPAD + H + 2 * MK_CONSUMERS;
  const size_t region = xfloats > (size_t)AF_END ? xfloats : (size_t)AF_END;
  return (size_t)n_stages * stage_bytes + 2 * MK_MAX_STAGES * 8 + region * 4;
}

}  // namespace flock
