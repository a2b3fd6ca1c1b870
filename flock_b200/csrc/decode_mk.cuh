// Persistent decode kernel: one cooperative launch per generated token.
//
// The kernel graph's kernels (k_embed, k_gemv, k_attn_decode_fast) become
// phases of one grid separated by grid barriers instead of kernel
// boundaries.  Each phase calls the same device functions with the same
// arguments the graph's launch would get (gemv_run, gemv_stage_x,
// attn_fast_item, gemv_argmax_finish), so logits and ids are bit-identical
// to the multi-kernel path.  Laid out for batch-1 latency on B200:
//
//  * grid = one CTA of 8 warps per SM (all co-resident: cooperative launch;
//    each phase function is compiled on its own, with up to 255 registers,
//    so no loop spills); in a GEMV phase every warp walks row groups across
//    the grid exactly as in a k_gemv launch of the same grid, reading weights
//    straight from global memory with its register lookahead;
//  * weights and KV rows do not depend on activations, so at the start of
//    each layer the grid issues L2 bulk prefetches of the NEXT layer's
//    weight and scale planes and KV rows (one 32 KiB piece per CTA at a
//    time): HBM streams layer l+1 while layer l computes out of L2;
//  * phases per layer: QKV (attn_norm fused) | attention (split-K, q/k norm +
//    RoPE + KV append fused, the last split of a group combines) | o_proj +
//    residual | gate/up (ffn_norm fused) + SwiGLU | down + residual; the
//    LM head and its argmax follow; layer 0's embedding is computed by every
//    CTA redundantly (CTA 0 publishes it as h) so it needs no barrier;
//  * the last CTA of the argmax writes the chosen id, its history slot and
//    the position.
//
// Grid barriers are bounded (global timer): on a timeout the kernel sets
// *err and every CTA stops working; the host reports the error.  No
// multicast loads are used.
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
  const void* kcache;  // prefetched only; attention reads through attn_args
  const void* vcache;
};

struct MkArgs {
  const MkLayer* layers;
  int n_layers;
  int H, nH, nKV, hd, F, vocab;
  int kv_bytes;  // bytes per cached key/value element: 4 (f32) or 2 (bf16)
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
  int64_t head_prefetch;  // bytes of the head's planes prefetched during the last layer
  // per-phase launch arguments built by the host, read from global memory by
  // every thread (a private copy per thread would be local-memory traffic):
  // gemv[4 * l + {0 QKV, 1 o_proj, 2 gate/up, 3 down}], gemv[4 * n_layers] the
  // head; attn[l] the attention phase of layer l
  const GemvArgs* gemv;
  const AttnFastArgs* attn_args;
  // optional phase trace: per CTA, mk_trace_stride(n_layers) entries of
  // global-timer nanoseconds -- stamps (start, embedded, then per layer and
  // phase: computed, released; head computed, done), then 6 zero words
  // (kept for the layout); nullptr when off
  unsigned long long* trace;
};

__host__ __device__ inline int mk_trace_stride(int n_layers) { return 10 + 10 * n_layers; }

constexpr int MK_THREADS = GEMV_THREADS;

FLOCK_DEV unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
FLOCK_DEV void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier over all CTAs.  Bounded; on timeout or a prior error anywhere
// it returns false and the caller stops working.
FLOCK_DEV bool grid_barrier(const MkArgs& a, unsigned& epoch) {
  __syncthreads();
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
  __syncthreads();
  return s_ok != 0;
}

// L2 prefetch of one layer's weight planes (qs, scales) and the K/V rows of
// keys 0..n_keys-1, spread over the grid in 32 KiB pieces (issue_prefetch).
// Planes above 24 MiB (the 8B shape's gate / up / down) stream on demand, so
// what is prefetched stays well inside the 126 MB L2.
FLOCK_DEV void mk_prefetch_layer(const MkArgs& a, int l, int n_keys) {
  const MkLayer& L = a.layers[l];
  const int rows[7] = {a.nH * a.hd, a.nKV * a.hd, a.nKV * a.hd, a.H, a.F, a.F, a.H};
  const int cols[7] = {a.H, a.H, a.H, a.nH * a.hd, a.H, a.H, a.F};
  PrefetchList pf = {};
  auto add = [&](const void* p, uint64_t bytes) {
    pf.ptr[pf.n] = reinterpret_cast<const uint8_t*>(p);
    pf.bytes[pf.n] = bytes & ~(uint64_t)15;
    if (++pf.n == 4) {
      issue_prefetch(pf);
      pf.n = 0;
    }
  };
  constexpr uint64_t kMax = 24ull << 20;
  for (int t = 0; t < 7; t++)
    if ((uint64_t)rows[t] * cols[t] <= kMax) add(L.qs[t], (uint64_t)rows[t] * cols[t]);
  for (int t = 0; t < 7; t++)
    if ((uint64_t)rows[t] * cols[t] <= kMax) add(L.sc[t], (uint64_t)rows[t] * L.sc_stride[t] * 2);
  const uint64_t kv = (uint64_t)n_keys * a.nKV * a.hd * a.kv_bytes;
  add(L.kcache, kv);
  add(L.vcache, kv);
  if (pf.n) issue_prefetch(pf);
}

// Runs a GEMV phase: the row-group walk of a k_gemv launch over this grid,
// x staged (and normalised) by gemv_stage_x.  One non-inlined function per
// shape: each phase gets the registers of its own loop, as its k_gemv
// launch would, instead of sharing the kernel's allocation.
template <int R, int EPI, int LA>
__device__ __noinline__ void mk_gemv_la(const GemvArgs* __restrict__ gp, const float* from,
                                        float* xs, float* gs, float* red, float& best_v,
                                        uint32_t& best_i) {
  const GemvArgs& g = *gp;
  gemv_run<QT_Q8, R, EPI, 1, LA>(g, 0, blockIdx.x, gridDim.x, xs, [&] {
    gemv_stage_x(g, 0, xs, gs, red, from);
    __syncthreads();
  }, best_v, best_i);
}
// `from`: the source row when it is not g->x (layer 0's embedded row in
// shared memory).
template <int R, int EPI>
FLOCK_DEV void mk_gemv(const GemvArgs* gp, const float* from, float* xs, float* gs, float* red,
                       float& best_v, uint32_t& best_i) {
  if ((gp->K / 32 + 31) / 32 >= 2)
    mk_gemv_la<R, EPI, 2>(gp, from, xs, gs, red, best_v, best_i);
  else
    mk_gemv_la<R, EPI, 1>(gp, from, xs, gs, red, best_v, best_i);
}

// The attention phase: work items (kv head, split) = (item / splits, item %
// splits), item = CTA, CTA + grid, ... (more items than CTAs when a long
// cache runs several splits per SM); all threads of the CTA work on each item.
__device__ __noinline__ void mk_attention(const AttnFastArgs* __restrict__ ap, int pos,
                                          float* att, bool* last) {
  const AttnFastArgs& aa = *ap;
  for (int item = blockIdx.x; item < aa.n_kv_heads * aa.splits; item += gridDim.x) {
    attn_fast_item(aa, item / aa.splits, item % aa.splits, pos, att, last, BlockSync{});
    __syncthreads();  // the next item reuses the shared tiles
  }
}

// Shared memory: x (padded) | gain staging | reduction scratch | CTA argmax
// slots | the embedded row; the attention phase reuses the region from 0.
struct MkShared {
  float* xs;
  float* gs;
  float* red;
  float* cta_val;
  uint32_t* cta_idx;
  float* raw;
  float* att;
};

static __global__ void __launch_bounds__(MK_THREADS, 1) k_decode_mk(const MkArgs a) {
  extern __shared__ __align__(128) float mk_smem[];
  const int kmax = max(a.H, max(a.nH * a.hd, a.F));
  MkShared sm;
  sm.xs = mk_smem;
  sm.gs = sm.xs + kmax / 32 * XPAD;
  sm.red = sm.gs + kmax;
  sm.cta_val = sm.red + 136;
  sm.cta_idx = reinterpret_cast<uint32_t*>(sm.cta_val + GEMV_WARPS);
  sm.raw = reinterpret_cast<float*>(sm.cta_idx + GEMV_WARPS);
  sm.att = mk_smem;
  __shared__ bool att_last;

  unsigned long long* tr =
      a.trace ? a.trace + (size_t)blockIdx.x * mk_trace_stride(a.n_layers) : nullptr;
  auto stamp = [&](int i) {
    if (tr && threadIdx.x == 0) tr[i] = globaltimer_ns();
  };
  stamp(0);
  if (tr && threadIdx.x == 0)
    for (int i = 4 + 10 * a.n_layers; i < mk_trace_stride(a.n_layers); i++) tr[i] = 0;
  const int pos = a.ctl[0] + a.ctl[1];  // this token's position
  const int token = a.ids[0];
  mk_prefetch_layer(a, 0, pos + 1);

  // layer 0's input: every CTA embeds the token itself (k_embed's
  // arithmetic); CTA 0 also publishes it as the residual stream h.
  if (token >= 0 && token < a.vocab) {
    for (int g = threadIdx.x; g < a.H / 4; g += MK_THREADS) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(a.embd_qs + (size_t)token * a.H + 4 * g);
      const float sc = scale_f16(a.embd_sc[(size_t)token * a.embd_sc_stride + g / 8]);
      float q0, q1, q2, q3;
      dec_i8x4(w, q0, q1, q2, q3);
      reinterpret_cast<float4*>(sm.raw)[g] =
          make_float4(fmul(q0, sc), fmul(q1, sc), fmul(q2, sc), fmul(q3, sc));
    }
  } else {
    for (int g = threadIdx.x; g < a.H / 4; g += MK_THREADS)
      reinterpret_cast<float4*>(sm.raw)[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < a.H; i += MK_THREADS) a.h[i] = sm.raw[i];
  stamp(1);

  float best_v = -FLT_MAX;
  uint32_t best_i = 0xFFFFFFFFu;
  unsigned epoch = 0;
  bool ok = true;
  for (int l = 0; l < a.n_layers && ok; l++) {
    if (l + 1 < a.n_layers) {
      mk_prefetch_layer(a, l + 1, pos + 1);
    } else if (a.head_prefetch > 0 && threadIdx.x == 0) {
      PrefetchList pf = {};
      pf.ptr[0] = a.head_qs;
      pf.bytes[0] = (uint64_t)a.head_prefetch & ~(uint64_t)15;
      pf.n = 1;
      issue_prefetch(pf);
    }
    const GemvArgs* G = a.gemv + 4 * l;
    // QKV (attn_norm fused): k_gemv<Q8, 2, STORE> over q | k | v
    mk_gemv<2, EPI_STORE>(G + 0, l == 0 ? sm.raw : nullptr, sm.xs, sm.gs, sm.red, best_v, best_i);
    stamp(2 + l * 10 + 0);
    if (!(ok = grid_barrier(a, epoch))) break;
    stamp(2 + l * 10 + 1);
    // attention (q/k norm + RoPE + KV append fused; the last split combines)
    mk_attention(a.attn_args + l, pos, sm.att, &att_last);
    stamp(2 + l * 10 + 2);
    if (!(ok = grid_barrier(a, epoch))) break;
    stamp(2 + l * 10 + 3);
    // o_proj + residual, in place on h
    mk_gemv<1, EPI_RESIDUAL>(G + 1, nullptr, sm.xs, sm.gs, sm.red, best_v, best_i);
    stamp(2 + l * 10 + 4);
    if (!(ok = grid_barrier(a, epoch))) break;
    stamp(2 + l * 10 + 5);
    // gate/up + SwiGLU (ffn_norm fused)
    mk_gemv<2, EPI_SWIGLU>(G + 2, nullptr, sm.xs, sm.gs, sm.red, best_v, best_i);
    stamp(2 + l * 10 + 6);
    if (!(ok = grid_barrier(a, epoch))) break;
    stamp(2 + l * 10 + 7);
    // down + residual, in place on h
    mk_gemv<1, EPI_RESIDUAL>(G + 3, nullptr, sm.xs, sm.gs, sm.red, best_v, best_i);
    stamp(2 + l * 10 + 8);
    ok = grid_barrier(a, epoch);
    stamp(2 + l * 10 + 9);
  }
  if (!ok) return;
  // output_norm + head + argmax: k_gemv<Q8, 2, ARGMAX> over the vocab
  const GemvArgs* hg = a.gemv + 4 * a.n_layers;
  mk_gemv<2, EPI_ARGMAX>(hg, nullptr, sm.xs, sm.gs, sm.red, best_v, best_i);
  stamp(2 + a.n_layers * 10);
  if (gemv_argmax_finish(*hg, best_v, best_i, sm.cta_val, sm.cta_idx) && threadIdx.x == 0) {
    // the chosen id (just written by this thread), its history slot, the position
    if (pos >= 0 && pos < a.hist_cap) a.hist[pos] = a.ids[0];
    a.ctl[0] = pos;
    a.ctl[1] = 1;
  }
  stamp(3 + a.n_layers * 10);
}

// Dynamic shared memory of a k_decode_mk launch.
inline size_t mk_smem_bytes(int H, int qw, int F) {
  const int kmax = H > qw ? (H > F ? H : F) : (qw > F ? qw : F);
  const size_t floats = (size_t)kmax / 32 * XPAD + kmax + 136 + 2 * GEMV_WARPS + H;
  const size_t region = floats > (size_t)AF_END ? floats : (size_t)AF_END;
  return region * 4 + 16;
}

}  // namespace flock
