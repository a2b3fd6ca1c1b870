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
};

constexpr int MK_CONSUMERS = 8;                   // consumer warps
constexpr int MK_THREADS = (MK_CONSUMERS + 1) * 32;
constexpr int MK_MAX_STAGES = 8;
constexpr uint64_t MK_WAIT_NS = 2000000000ull;    // a wait gives up after 2 s
constexpr uint32_t MK_MAX_POLLS = 1u << 26;       // backstop on the poll count

// ------------------------------------------------------------- primitives
FLOCK_DEV uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
FLOCK_DEV void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
FLOCK_DEV void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes) : "memory");
}
FLOCK_DEV void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
FLOCK_DEV bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
FLOCK_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: false after MK_WAIT_NS of global time (or MK_MAX_POLLS polls),
// or as soon as *err is set when `watch_err`.
FLOCK_DEV bool mbar_wait(uint64_t* b, uint32_t parity, const int* err, bool watch_err = true) {
  uint64_t t0 = 0;
  for (uint32_t i = 0; i < MK_MAX_POLLS; i++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 63) == 63) {
      if (watch_err && *(volatile const int*)err) return false;
      const uint64_t now = globaltimer_ns();
      if (!t0) t0 = now;
      else if (now - t0 > MK_WAIT_NS) return false;
    }
  }
  return false;
}
FLOCK_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
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
      if (now - t0 > MK_WAIT_NS || i >= MK_MAX_POLLS) {
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

// x for the next phase into the padded shared layout, RMSNorm fused when
// `gain` is given: the same one-round-trip staging and exact ops_ref.ts:20
// order as rmsnorm_to_smem, synchronised over the consumer warps only.
// `src` may point to global or shared memory.
FLOCK_DEV void mk_stage_x(const float* src, int K, const float* gain, float eps, float* xs,
                          float* gs, float* red) {
  const int t = threadIdx.x;
  for (int i = t; i < K / 4; i += MK_CONSUMERS * 32) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    reinterpret_cast<float4*>(xs)[(i >> 3) * (XPAD / 4) + (i & 7)] = v;
    if (gain) reinterpret_cast<float4*>(gs)[i] = reinterpret_cast<const float4*>(gain)[i];
  }
  consumers_sync();
  if (!gain) return;
  if (t < 128) {
    float acc = 0.0f;
    for (int i = t; i < K; i += 128) {
      const float v = xs[xpad(i)];
      acc = ffma(v, v, acc);
    }
    red[t] = acc;
  }
  consumers_sync();
  if (t < 64) red[t] = fadd(red[t], red[t + 64]);
  consumers_sync();
  if (t < 32) {
    float v = fadd(red[t], red[t + 32]);
    v = warp_tree_sum(v);
    if (t == 0) red[128] = rsqrt_f64r(fadd(fdiv(v, (float)K), eps));
  }
  consumers_sync();
  const float scale = red[128];
  for (int i = t; i < K; i += MK_CONSUMERS * 32)
    xs[xpad(i)] = fmul(fmul(xs[xpad(i)], scale), gs[i]);
  consumers_sync();
}

// One row held in shared memory against the staged x: the reference's
// coop(64) order (lane plays logical lanes lane and lane+32), block 0 of x
// from registers, the rest from the padded shared copy.  Lane 0 gets y.
FLOCK_DEV float mk_row_dot(const uint8_t* rq, const uint16_t* rs, int nb, const float4 (&xr0)[8],
                           const float4* xs4, int lane) {
  float accA = 0.0f, accB = 0.0f;
  const int M = (nb + 31) / 32;
  for (int m = 0; m < M; m++) {
    const int b = lane + 32 * m;
    if (b >= nb) break;
    BlockW<QT_Q8> bw;
    load_block_smem(bw, rq, rs, b);
    if (m == 0)
      accA = fold_block<QT_Q8>(bw, xr0, accA);
    else if (m & 1)
      accB = fold_block<QT_Q8>(bw, xs4 + b * (XPAD / 4), accB);
    else
      accA = fold_block<QT_Q8>(bw, xs4 + b * (XPAD / 4), accA);
  }
  return warp_tree_sum(fadd(accA, accB));
}

struct MkShared {
  float* xs;      // padded x
  float* gs;      // gain staging
  float* red;     // [136]
  float* raw;     // [H] embedded row (layer 0)
  float* wv;      // [MK_CONSUMERS] argmax values
  uint32_t* wi;   // [MK_CONSUMERS] argmax indices
  float* att;     // AF_END floats for the attention phase (aliases the above)
};

// A GEMV phase over this CTA's chunks.  Returns false if a wait gave up.
template <int P>
FLOCK_DEV void mk_gemv_phase(const MkArgs& a, int layer, uint8_t* ring, uint64_t* full,
                             uint64_t* empty, int& cidx, const MkShared& sm, float& best_v,
                             uint32_t& best_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float4* xs4 = reinterpret_cast<const float4*>(sm.xs);
  float4 xr0[8];
  {
    const PhaseGeo g = phase_geo(a, P);
    const int nb = g.K / 32;
#pragma unroll
    for (int j = 0; j < 8; j++)
      xr0[j] = lane < nb ? xs4[lane * (XPAD / 4) + j] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const MkLayer* L = P == PH_HEAD ? nullptr : a.layers + layer;
  for_each_chunk(a, P, [&](const Chunk& c) {
    const int st = cidx % a.n_stages;
    if (!mbar_wait(&full[st], (uint32_t)((cidx / a.n_stages) & 1), a.err)) atomicCAS(a.err, 0, 1);
    const uint8_t* stage = ring + (size_t)st * a.stage_bytes;
    const int nb = c.K / 32;
    const int scs = (nb + 7) / 8 * 8;
    const int nsrc = P == PH_GU ? 2 : 1;
    const uint32_t qbytes = (uint32_t)c.rows * c.K;
    const uint8_t* q0 = stage;
    const uint8_t* q1 = stage + qbytes;
    const uint16_t* s0 = reinterpret_cast<const uint16_t*>(stage + nsrc * qbytes);
    const uint16_t* s1 = s0 + (size_t)c.rows * scs;
    for (int u = warp; u < c.rows; u += MK_CONSUMERS) {
      const int row = c.row0 + u;
      const float y = mk_row_dot(q0 + (size_t)u * c.K, s0 + (size_t)u * scs, nb, xr0, xs4, lane);
      if (P == PH_GU) {
        const float yu = mk_row_dot(q1 + (size_t)u * c.K, s1 + (size_t)u * scs, nb, xr0, xs4, lane);
        if (lane == 0) {
          // ops_ref.ts:103 swigluRef: fr(fr(g / fr(1 + fr(exp(-g)))) * up)
          const float e = exp_f64r(-y);
          a.act[row] = fmul(fdiv(y, fadd(1.0f, e)), yu);
        }
      } else if (lane == 0) {
        if (P == PH_QKV) {
          float* dst = c.seg == 0 ? a.q : (c.seg == 1 ? a.k : a.v);
          dst[row] = y;
        } else if (P == PH_O || P == PH_DOWN) {
          a.h[row] = fadd(a.h[row], y);
        } else if (P == PH_HEAD) {
          a.logits[row] = y;
          if (am_better(y, (uint32_t)row, best_v, best_i)) {
            best_v = y;
            best_i = (uint32_t)row;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    cidx++;
  });
  (void)L;
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
  sm.red = sm.gs + a.H;
  sm.raw = sm.red + 136;
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

  const int pos = a.ctl[0] + a.ctl[1];  // this token's position
  const int token = a.ids[0];

  if (warp == MK_CONSUMERS) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int cidx = 0;
      bool stop = false;
      auto produce = [&](int layer, int p) {
        for_each_chunk(a, p, [&](const Chunk& c) {
          if (stop) return;
          const int st = cidx % a.n_stages;
          if (cidx >= a.n_stages &&
              !mbar_wait(&empty[st], (uint32_t)(((cidx / a.n_stages) - 1) & 1), a.err)) {
            stop = true;
            return;
          }
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

    bool ok = true;
    for (int l = 0; l < a.n_layers && ok; l++) {
      const MkLayer& L = a.layers[l];
      // QKV (attn_norm fused)
      mk_stage_x(l == 0 ? sm.raw : a.h, a.H, L.attn_norm, a.eps, sm.xs, sm.gs, sm.red);
      mk_gemv_phase<PH_QKV>(a, l, ring, full, empty, cidx, sm, best_v, best_i);
      if (!(ok = grid_barrier(a, epoch))) break;
      // attention (q/k norm + RoPE + KV append fused)
      aa.q_norm = L.q_norm;
      aa.k_norm = L.k_norm;
      aa.kcache = L.kcache;
      aa.vcache = L.vcache;
      if ((int)blockIdx.x < a.nKV * a.splits)
        attn_fast_item(aa, blockIdx.x / a.splits, blockIdx.x % a.splits, pos, sm.att, &att_last,
                       ConsumerSync{});
      if (!(ok = grid_barrier(a, epoch))) break;
      // o_proj + residual
      mk_stage_x(a.attn, a.nH * a.hd, nullptr, a.eps, sm.xs, sm.gs, sm.red);
      mk_gemv_phase<PH_O>(a, l, ring, full, empty, cidx, sm, best_v, best_i);
      if (!(ok = grid_barrier(a, epoch))) break;
      // gate/up + SwiGLU (ffn_norm fused)
      mk_stage_x(a.h, a.H, L.ffn_norm, a.eps, sm.xs, sm.gs, sm.red);
      mk_gemv_phase<PH_GU>(a, l, ring, full, empty, cidx, sm, best_v, best_i);
      if (!(ok = grid_barrier(a, epoch))) break;
      // down + residual
      mk_stage_x(a.act, a.F, nullptr, a.eps, sm.xs, sm.gs, sm.red);
      mk_gemv_phase<PH_DOWN>(a, l, ring, full, empty, cidx, sm, best_v, best_i);
      ok = grid_barrier(a, epoch);
    }
    if (ok) {
    // output_norm + head + argmax
    mk_stage_x(a.h, a.H, a.out_norm, a.eps, sm.xs, sm.gs, sm.red);
    mk_gemv_phase<PH_HEAD>(a, 0, ring, full, empty, cidx, sm, best_v, best_i);
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
    if (last && threadIdx.x == 0) {
      __threadfence();
      float bv = -FLT_MAX;
      uint32_t bi = 0xFFFFFFFFu;
      for (int i = 0; i < (int)gridDim.x; i++) {
        const float v = ((volatile float*)a.am_val)[i];
        const uint32_t ix = ((volatile uint32_t*)a.am_idx)[i];
        if (am_better(v, ix, bv, bi)) {
          bv = v;
          bi = ix;
        }
      }
      *a.am_best_val = bv;
      a.ids[0] = (int32_t)bi;
      if (pos >= 0 && pos < a.hist_cap) a.hist[pos] = (int32_t)bi;
      a.ctl[0] = pos;
      a.ctl[1] = 1;
      *a.am_count = 0;
    }
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
  const size_t xfloats = (size_t)kmax / 32 * XPAD + H + 136 + H + 2 * MK_CONSUMERS;
  const size_t region = xfloats > (size_t)AF_END ? xfloats : (size_t)AF_END;
  return (size_t)n_stages * stage_bytes + 2 * MK_MAX_STAGES * 8 + region * 4;
}

}  // namespace flock
