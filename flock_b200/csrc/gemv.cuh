// Q8_0 / Q4_0 dequantising matvec for B200, in the reference's exact f32 order.
//
// What it computes (kernels/q8_coop.wgsl:76, kernels/q4_coop.wgsl:48, CPU
// model kernels/lib.ts:213 matmulF32 with coop(64)): for row r,
//   logical lane l in [0,64) walks blocks b = l, l+64, l+128, ... and folds
//   scale_b * (dot4(q[8g..8g+3], x) + dot4(q[8g+4..8g+7], x)) into its own
//   accumulator for g = 0..3 (Q4_0: q[4g..4g+3] / q[4g+16..4g+19]);
//   the 64 accumulators are then summed by the pairwise tree.
// The result is bit-identical to cpuMatmulQ8F32(coop(64)) / cpuMatmulQ4F32.
//
// How it is laid out on the GPU (not how the WGSL is): one warp owns a group
// of R rows; lane t of the warp plays logical lanes t and t+32, i.e. blocks
// t + 32m with m even (lane t) and m odd (lane t+32).  A warp therefore reads
// each row as contiguous 1 KiB runs of qs -- fully coalesced 128-bit streams
// straight from HBM -- and the tree's first level (stride 32) is a register
// add, the remaining five are warp shuffles.  x lives in shared memory (with
// the attn/ffn/output RMSNorm optionally fused into the load) and the first
// MX of each thread's x blocks are held in registers for the whole kernel.
//
// Launch: persistent-style grid of <= 2 CTAs per SM; each warp strides over
// row groups.  Before griddepcontrol.wait the kernel only touches weights: it
// issues the L2 prefetch list for the NEXT kernel and the loads of its own
// first row group, so both overlap the previous kernel's tail.
#pragma once
#include "common.cuh"

namespace flock {

enum { QT_Q8 = 0, QT_Q4 = 1 };
enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

struct GemvSeg {
  const uint8_t* qs;   // Q8: [rows][K] int8; Q4: [rows][K/32][16] nibble pairs
  const uint16_t* sc;  // [rows][sc_stride] f16 scales
  float* out;          // [n_tokens][out_stride]
  int rows;
  int sc_stride;
  int out_stride;
};

struct GemvArgs {
  GemvSeg seg[3];
  int nseg;
  int K;
  int n_tokens;
  // input: x [n_tokens][x_stride] or rmsnorm(norm_src[t], norm_gain)
  const float* x;
  int x_stride;
  const float* norm_gain;  // non-null -> fused rmsnorm prologue (ops_ref.ts:20, WG=128)
  float eps;
  // epilogue inputs
  const float* res;  // EPI_RESIDUAL: [n_tokens][res_stride]
  int res_stride;
  // EPI_ARGMAX: per-CTA partials, arrival counter, final (value, index)
  float* am_val;
  uint32_t* am_idx;
  uint32_t* am_count;
  float* am_best_val;
  int32_t* am_best_idx;
  int am_row_offset;  // added to the reported index (a row shard's first row)
  // step control {pos, n_last}: advanced once by CTA (0,0) when non-null
  int* ctl;
  int ctl_n;
  PrefetchList pf;
};

// Weights of one row in one 32-weight block, as loaded for one thread.
template <int QT>
struct BlockW;
template <>
struct BlockW<QT_Q8> {
  uint4 w0, w1;
  uint16_t s;
};
template <>
struct BlockW<QT_Q4> {
  uint4 w;
  uint16_t s;
};

template <int QT>
FLOCK_DEV void load_block(BlockW<QT>& bw, const GemvSeg& sg, int row, int b, int K);
template <>
FLOCK_DEV void load_block<QT_Q8>(BlockW<QT_Q8>& bw, const GemvSeg& sg, int row, int b, int K) {
  const uint8_t* p = sg.qs + (size_t)row * K + (size_t)b * 32;
  bw.w0 = ldg_stream(p);
  bw.w1 = ldg_stream(p + 16);
  bw.s = __ldg(sg.sc + (size_t)row * sg.sc_stride + b);
}
template <>
FLOCK_DEV void load_block<QT_Q4>(BlockW<QT_Q4>& bw, const GemvSeg& sg, int row, int b, int K) {
  const uint8_t* p = sg.qs + ((size_t)row * (K / 32) + b) * 16;
  bw.w = ldg_stream(p);
  bw.s = __ldg(sg.sc + (size_t)row * sg.sc_stride + b);
}

// Fold one block into acc in the reference order.  xb points at the block's
// 32 x values as 8 float4 (registers, or a padded shared-memory row).
template <int QT>
FLOCK_DEV float fold_block(const BlockW<QT>& bw, const float4* xb, float acc);
template <>
FLOCK_DEV float fold_block<QT_Q8>(const BlockW<QT_Q8>& bw, const float4* xb, float acc) {
  const float s = scale_f16(bw.s);
  const uint32_t w[8] = {bw.w0.x, bw.w0.y, bw.w0.z, bw.w0.w, bw.w1.x, bw.w1.y, bw.w1.z, bw.w1.w};
#pragma unroll
  for (int g = 0; g < 4; g++) {
    float a0, a1, a2, a3, c0, c1, c2, c3;
    dec_i8x4(w[2 * g], a0, a1, a2, a3);
    dec_i8x4(w[2 * g + 1], c0, c1, c2, c3);
    const float4 xa = xb[2 * g], xc = xb[2 * g + 1];
    float d0 = dot4(a0, a1, a2, a3, xa.x, xa.y, xa.z, xa.w);
    float d1 = dot4(c0, c1, c2, c3, xc.x, xc.y, xc.z, xc.w);
    acc = ffma(s, fadd(d0, d1), acc);
  }
  return acc;
}
template <>
FLOCK_DEV float fold_block<QT_Q4>(const BlockW<QT_Q4>& bw, const float4* xb, float acc) {
  const float s = scale_f16(bw.s);
  const uint32_t w[4] = {bw.w.x, bw.w.y, bw.w.z, bw.w.w};
#pragma unroll
  for (int g = 0; g < 4; g++) {
    float a0, a1, a2, a3, c0, c1, c2, c3;
    dec_nib4(w[g] & 0x0F0F0F0Fu, a0, a1, a2, a3);
    dec_nib4((w[g] >> 4) & 0x0F0F0F0Fu, c0, c1, c2, c3);
    const float4 xa = xb[g], xc = xb[4 + g];  // cols 4g.. and 16+4g..
    float d0 = dot4(a0, a1, a2, a3, xa.x, xa.y, xa.z, xa.w);
    float d1 = dot4(c0, c1, c2, c3, xc.x, xc.y, xc.z, xc.w);
    acc = ffma(s, fadd(d0, d1), acc);
  }
  return acc;
}

// x lives in shared memory with each 32-float block padded to 36 floats, so
// lane l reading block l (float4 at a time) touches distinct banks.
constexpr int XPAD = 36;
FLOCK_DEV int xpad(int i) { return (i >> 5) * XPAD + (i & 31); }

// The packed-pair layout the f32x2 folds (persistent decode kernel) read:
// inside each padded 32-float
// block, u64 element 4g + k holds the two x values that weight pair k of
// group g multiplies -- Q8_0 (x[8g+k], x[8g+4+k]), Q4_0 (x[4g+k],
// x[16+4g+k]) -- so a 128-bit shared read yields two f32x2 operands.
template <int QT>
FLOCK_DEV int xperm(int i) {
  const int j = i & 31;
  const int p = QT == QT_Q8 ? (j & ~7) + 2 * (j & 3) + ((j >> 2) & 1) : 2 * (j & 15) + (j >> 4);
  return (i >> 5) * XPAD + p;
}

// n floats of src (global or shared) into xs in the packed-pair layout.
template <int QT>
FLOCK_DEV void stage_x_packed(const float* src, int n, float* xs, int tid, int nthreads) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  for (int i = tid; i < n / 8; i += nthreads) {
    const int b = i >> 2, q = i & 3;
    // Q8_0: the 8-float group i; Q4_0: floats 4q.. and 16+4q.. of block b
    const float4 lo = QT == QT_Q8 ? s4[2 * i] : s4[b * 8 + q];
    const float4 hi = QT == QT_Q8 ? s4[2 * i + 1] : s4[b * 8 + 4 + q];
    float4* d = reinterpret_cast<float4*>(xs + b * XPAD + q * 8);
    d[0] = make_float4(lo.x, hi.x, lo.y, hi.y);
    d[1] = make_float4(lo.z, hi.z, lo.w, hi.w);
  }
}

// Block b of packed x as 16 pairs.
FLOCK_DEV void load_pairs(const float* xs, int b, uint64_t (&xp)[16]) {
  const ulonglong2* q = reinterpret_cast<const ulonglong2*>(xs + b * XPAD);
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const ulonglong2 v = q[j];
    xp[2 * j] = v.x;
    xp[2 * j + 1] = v.y;
  }
}

// fold_block on packed pairs: the two dot4 chains of a group run as the
// halves of one f32x2 chain (each half rounds as the scalar instruction),
// then acc = fma(scale, d0 + d1, acc) -- fold_block's arithmetic exactly.
template <int QT>
FLOCK_DEV float fold_block_packed(const BlockW<QT>& bw, const uint64_t (&xp)[16], float acc);
template <>
FLOCK_DEV float fold_block_packed<QT_Q8>(const BlockW<QT_Q8>& bw, const uint64_t (&xp)[16],
                                         float acc) {
  const float s = scale_f16(bw.s);
  const uint32_t w[8] = {bw.w0.x, bw.w0.y, bw.w0.z, bw.w0.w, bw.w1.x, bw.w1.y, bw.w1.z, bw.w1.w};
  const uint64_t k2 = pack2(8388736.0f, 8388736.0f);  // 2^23 + 128
#pragma unroll
  for (int g = 0; g < 4; g++) {
    const uint32_t ua = w[2 * g] ^ 0x80808080u, uc = w[2 * g + 1] ^ 0x80808080u;
    uint64_t q[4];
#pragma unroll
    for (int k = 0; k < 4; k++)
      q[k] = fsub2(pack2(__uint_as_float(__byte_perm(ua, 0x4B000000u, 0x7540u + k)),
                         __uint_as_float(__byte_perm(uc, 0x4B000000u, 0x7540u + k))),
                   k2);
    uint64_t d = fmul2(q[0], xp[4 * g]);
    d = ffma2(q[1], xp[4 * g + 1], d);
    d = ffma2(q[2], xp[4 * g + 2], d);
    d = ffma2(q[3], xp[4 * g + 3], d);
    const float2 dd = unpack2(d);
    acc = ffma(s, fadd(dd.x, dd.y), acc);
  }
  return acc;
}
template <>
FLOCK_DEV float fold_block_packed<QT_Q4>(const BlockW<QT_Q4>& bw, const uint64_t (&xp)[16],
                                         float acc) {
  const float s = scale_f16(bw.s);
  const uint32_t w[4] = {bw.w.x, bw.w.y, bw.w.z, bw.w.w};
  const uint64_t k2 = pack2(8388616.0f, 8388616.0f);  // 2^23 + 8
#pragma unroll
  for (int g = 0; g < 4; g++) {
    const uint32_t lo = w[g] & 0x0F0F0F0Fu, hi = (w[g] >> 4) & 0x0F0F0F0Fu;
    uint64_t q[4];
#pragma unroll
    for (int k = 0; k < 4; k++)
      q[k] = fsub2(pack2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u + k)),
                         __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u + k))),
                   k2);
    uint64_t d = fmul2(q[0], xp[4 * g]);
    d = ffma2(q[1], xp[4 * g + 1], d);
    d = ffma2(q[2], xp[4 * g + 2], d);
    d = ffma2(q[3], xp[4 * g + 3], d);
    const float2 dd = unpack2(d);
    acc = ffma(s, fadd(dd.x, dd.y), acc);
  }
  return acc;
}

// kernels/argmax.wgsl:57 better(): strictly larger, or equal with lower index.
FLOCK_DEV bool am_better(float va, uint32_t ia, float vb, uint32_t ib) {
  return va > vb || (va == vb && ia < ib);
}

// Fused RMSNorm prologue, exact ops_ref.ts:20 order with WG = 128:
// part[t] = serial fma over i = t, t+128, ...; pairwise tree over 128;
// scale = fr(1/sqrt(fr(fr(sum/n) + eps))); y = fr(fr(x*scale)*g).
// x and the gain are staged into shared memory with ONE round trip of
// 128-bit loads (all issued before any is consumed); the rest runs on chip.
// Called by all GEMV_THREADS threads; leaves y in xs in layout LAYOUT
// (xidx: 0 padded, 1 / 2 the Q8_0 / Q4_0 packed-pair layouts).
template <int LAYOUT>
FLOCK_DEV int xidx(int i) {
  return LAYOUT == 0 ? xpad(i) : xperm<LAYOUT - 1>(i);
}
template <int LAYOUT = 0>
FLOCK_DEV void rmsnorm_to_smem(const float* __restrict__ src, const float* __restrict__ gain,
                               int n, float eps, float* xs, float* gs, float* red) {
  const int t = threadIdx.x;
  if (n % 128 == 0 && n <= 1024) {
    // thread t < 128 loads the elements of its own WG = 128 partial (t,
    // t + 128, ...) and folds them in registers; the tree's two cross-warp
    // levels run in one step, (r[l] + r[l+64]) + (r[l+32] + r[l+96]); the
    // normalised values are written once -- the same operations in the same
    // order as the general path below, with two fewer CTA barriers
    const int E = n / 128;
    float v[8], g[8];
    if (t < 128) {
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        v[j] = j < E ? src[t + 128 * j] : 0.0f;
        g[j] = j < E ? gain[t + 128 * j] : 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j < E) acc = ffma(v[j], v[j], acc);
      red[t] = acc;
    }
    __syncthreads();
    if (t < 32) {
      float s = fadd(fadd(red[t], red[t + 64]), fadd(red[t + 32], red[t + 96]));
      s = warp_tree_sum(s);
      if (t == 0) red[128] = rsqrt_f64r(fadd(fdiv(s, (float)n), eps));
    }
    __syncthreads();
    if (t < 128) {
      const float scale = red[128];
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j < E) xs[xidx<LAYOUT>(t + 128 * j)] = fmul(fmul(v[j], scale), g[j]);
    }
    return;
  }
  const float4* s4 = reinterpret_cast<const float4*>(src);
  const float4* g4 = reinterpret_cast<const float4*>(gain);
#pragma unroll 4
  for (int i = t; i < n / 4; i += GEMV_THREADS) {
    const float4 v = s4[i];
    const float4 g = g4[i];
    if (LAYOUT == 0) {
      reinterpret_cast<float4*>(xs)[(i >> 3) * (XPAD / 4) + (i & 7)] = v;
    } else {
      xs[xidx<LAYOUT>(4 * i)] = v.x;
      xs[xidx<LAYOUT>(4 * i + 1)] = v.y;
      xs[xidx<LAYOUT>(4 * i + 2)] = v.z;
      xs[xidx<LAYOUT>(4 * i + 3)] = v.w;
    }
    reinterpret_cast<float4*>(gs)[i] = g;
  }
  __syncthreads();
  if (t < 128) {
    float acc = 0.0f;
    for (int i = t; i < n; i += 128) {
      const float v = xs[xidx<LAYOUT>(i)];
      acc = ffma(v, v, acc);
    }
    red[t] = acc;
  }
  __syncthreads();
  if (t < 64) red[t] = fadd(red[t], red[t + 64]);
  __syncthreads();
  if (t < 32) {
    float v = fadd(red[t], red[t + 32]);
    v = warp_tree_sum(v);
    if (t == 0) red[128] = rsqrt_f64r(fadd(fdiv(v, (float)n), eps));
  }
  __syncthreads();
  const float scale = red[128];
  for (int i = t; i < n; i += GEMV_THREADS)
    xs[xidx<LAYOUT>(i)] = fmul(fmul(xs[xidx<LAYOUT>(i)], scale), gs[i]);
}

// The R rows a row group covers.
template <int R>
struct Rows {
  int seg[R], row[R];
  bool ok[R];
};

template <int R, int EPI>
FLOCK_DEV void rows_of(const GemvArgs& a, int g, Rows<R>& rs) {
  if (EPI == EPI_SWIGLU) {
    // R/2 gate rows (segment 0) and the same R/2 up rows (segment 1)
    const int r0 = g * (R / 2);
#pragma unroll
    for (int r = 0; r < R; r++) {
      rs.seg[r] = r < R / 2 ? 0 : 1;
      rs.row[r] = r0 + (r % (R / 2));
      rs.ok[r] = rs.row[r] < a.seg[0].rows;
    }
  } else {
    int s = 0, row0 = 0;
#pragma unroll
    for (int q = 0; q < 3; q++) {
      if (q >= a.nseg) break;
      const int ng = (a.seg[q].rows + R - 1) / R;
      if (g < ng) {
        s = q;
        row0 = g * R;
        break;
      }
      g -= ng;
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      rs.seg[r] = s;
      rs.row[r] = row0 + r;
      rs.ok[r] = rs.row[r] < a.seg[s].rows;
    }
  }
}

// MX: how many of each thread's x blocks (lane + 32m, m < MX) stay in
// registers; the rest are read from shared memory.
// LA: steps in flight ahead of the one being folded (1, or 2 for long rows,
// where each warp walks several column blocks per row and one step of
// lookahead leaves HBM latency exposed).
//
// gemv_run: the matvec of CTA `cta` of `n_ctas` (warps stride over row groups
// across the CTAs) for token `tok`.  The first step's weight loads are issued,
// then `pre()` runs -- it must leave x (padded layout) in xs and synchronise
// the block -- then the rows are folded and the epilogue applied.  EPI_ARGMAX
// leaves this thread's best (value, index) in best_v / best_i.
// PK != 0: x is staged in the packed-pair layout (pre() must do so:
// gemv_stage_x with layout 1 + QT) and blocks fold with fold_block_packed --
// the same arithmetic in about a quarter fewer instructions.  PK 1: rows of
// one block per lane (K <= 1024), whose pairs stay in registers; PK 2: any
// row length, the pairs read from shared memory per step.
template <int QT, int R, int EPI, int MX, int LA, int PK = 0, class Pre>
FLOCK_DEV void gemv_run(const GemvArgs& a, int tok, int cta, int n_ctas, const float* xs,
                        Pre&& pre, float& best_v, uint32_t& best_i) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nb = a.K / 32;
  const int M = (nb + 31) / 32;

  int n_groups;
  if (EPI == EPI_SWIGLU) {
    n_groups = (a.seg[0].rows + R / 2 - 1) / (R / 2);
  } else {
    n_groups = 0;
    for (int s = 0; s < a.nseg; s++) n_groups += (a.seg[s].rows + R - 1) / R;
  }
  const int nwarps = n_ctas * GEMV_WARPS;

  // The warp walks steps (g, m): row group g = gwarp, gwarp + nwarps, ...,
  // column block m = 0..M-1.  Weights do not depend on any earlier kernel,
  // so the first step's loads are issued before griddepcontrol.wait.
  int g = cta * GEMV_WARPS + warp, m = 0;
  bool have = g < n_groups;
  Rows<R> rs;
  BlockW<QT> cur[R];
  if (have) {
    rows_of<R, EPI>(a, g, rs);
    if (lane < nb) {
#pragma unroll
      for (int r = 0; r < R; r++)
        if (rs.ok[r]) load_block<QT>(cur[r], a.seg[rs.seg[r]], rs.row[r], lane, a.K);
    }
  }
  // LA = 2: the following step is in flight too
  int g1 = g, m1 = 0;
  bool have1 = false;
  Rows<R> rs1 = rs;
  BlockW<QT> nx1[R];
  if (LA == 2) {
    m1 = m + 1;
    if (m1 == M) {
      m1 = 0;
      g1 = g + nwarps;
    }
    have1 = have && g1 < n_groups;
    if (have1 && m1 == 0) rows_of<R, EPI>(a, g1, rs1);
    const int b1 = lane + 32 * m1;
    if (have1 && b1 < nb) {
#pragma unroll
      for (int r = 0; r < R; r++)
        if (rs1.ok[r]) load_block<QT>(nx1[r], a.seg[rs1.seg[r]], rs1.row[r], b1, a.K);
    }
  }

  pre();

  const float4* xs4 = reinterpret_cast<const float4*>(xs);
  float4 xr[PK ? 1 : MX][8];
  uint64_t xp[PK == 1 ? 16 : 1];
  if (PK == 1) {
    if (lane < nb) {
      load_pairs(xs, lane, reinterpret_cast<uint64_t(&)[16]>(xp));
    } else {
#pragma unroll
      for (int j = 0; j < (PK == 1 ? 16 : 1); j++) xp[j] = 0;
    }
  } else if (PK == 0) {
#pragma unroll
    for (int mm = 0; mm < MX; mm++) {
      const int b = lane + 32 * mm;
#pragma unroll
      for (int j = 0; j < 8; j++)
        xr[mm][j] = (b < nb) ? xs4[b * (XPAD / 4) + j] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  float accA[R], accB[R];
#pragma unroll
  for (int r = 0; r < R; r++) accA[r] = accB[r] = 0.0f;
  // EPI_RESIDUAL: lane 0 loads the group's residual rows when the group
  // starts, so the round trip overlaps the fold instead of following it
  float resv[EPI == EPI_RESIDUAL ? R : 1];

  while (have) {
    if (EPI == EPI_RESIDUAL && m == 0 && lane == 0) {
#pragma unroll
      for (int r = 0; r < R; r++)
        resv[r] = rs.ok[r] ? a.res[(size_t)tok * a.res_stride + rs.row[r]] : 0.0f;
    }
    // issue the loads of the step LA ahead before folding this one
    const int gb = LA == 2 ? g1 : g, mb = LA == 2 ? m1 : m;
    int g2 = gb, m2 = mb + 1;
    if (m2 == M) {
      m2 = 0;
      g2 = gb + nwarps;
    }
    const bool have2 = (LA == 2 ? have1 : true) && g2 < n_groups;
    Rows<R> rs2 = LA == 2 ? rs1 : rs;
    if (have2 && m2 == 0) rows_of<R, EPI>(a, g2, rs2);
    BlockW<QT> nxt[R];
    const int b2 = lane + 32 * m2;
    if (have2 && b2 < nb) {
#pragma unroll
      for (int r = 0; r < R; r++)
        if (rs2.ok[r]) load_block<QT>(nxt[r], a.seg[rs2.seg[r]], rs2.row[r], b2, a.K);
    }

    const int b = lane + 32 * m;
    if (b < nb) {
      auto fold_all = [&](const float4* xb) {
#pragma unroll
        for (int r = 0; r < R; r++) {
          if (!rs.ok[r]) continue;
          if (m & 1)
            accB[r] = fold_block<QT>(cur[r], xb, accB[r]);
          else
            accA[r] = fold_block<QT>(cur[r], xb, accA[r]);
        }
      };
      if (PK == 1) {  // the lane's only block (M == 1): pairs held in registers
#pragma unroll
        for (int r = 0; r < R; r++)
          if (rs.ok[r])
            accA[r] = fold_block_packed<QT>(cur[r], reinterpret_cast<uint64_t(&)[16]>(xp), accA[r]);
      } else if (PK == 2) {
        uint64_t xq[16];
        load_pairs(xs, b, xq);
#pragma unroll
        for (int r = 0; r < R; r++) {
          if (!rs.ok[r]) continue;
          if (m & 1)
            accB[r] = fold_block_packed<QT>(cur[r], xq, accB[r]);
          else
            accA[r] = fold_block_packed<QT>(cur[r], xq, accA[r]);
        }
      } else if (m < MX) {
        fold_all(xr[MX >= 2 && m == 1 ? 1 : 0]);
      } else {
        fold_all(xs4 + b * (XPAD / 4));
      }
    }

    if (m == M - 1) {
      float y[R];
#pragma unroll
      for (int r = 0; r < R; r++) {
        y[r] = warp_tree_sum(fadd(accA[r], accB[r]));
        accA[r] = accB[r] = 0.0f;
      }
      if (lane == 0) {
        if (EPI == EPI_SWIGLU) {
#pragma unroll
          for (int r = 0; r < R / 2; r++) {
            if (!rs.ok[r]) continue;
            // ops_ref.ts:103 swigluRef: fr(fr(g / fr(1 + fr(exp(-g)))) * up)
            const float gt = y[r], up = y[r + R / 2];
            const float e = exp_f64r(-gt);
            const float sg = fdiv(gt, fadd(1.0f, e));
            a.seg[0].out[(size_t)tok * a.seg[0].out_stride + rs.row[r]] = fmul(sg, up);
          }
        } else {
#pragma unroll
          for (int r = 0; r < R; r++) {
            if (!rs.ok[r]) continue;
            const GemvSeg& sg = a.seg[rs.seg[r]];
            float v = y[r];
            if (EPI == EPI_RESIDUAL) v = fadd(resv[EPI == EPI_RESIDUAL ? r : 0], v);
            sg.out[(size_t)tok * sg.out_stride + rs.row[r]] = v;
            if (EPI == EPI_ARGMAX) {
              const uint32_t idx = (uint32_t)(rs.row[r] + a.am_row_offset);
              if (am_better(v, idx, best_v, best_i)) {
                best_v = v;
                best_i = idx;
              }
            }
          }
        }
      }
    }

    if (LA == 2) {
#pragma unroll
      for (int r = 0; r < R; r++) {
        cur[r] = nx1[r];
        nx1[r] = nxt[r];
      }
      g = g1;
      m = m1;
      rs = rs1;
      have = have1;
      g1 = g2;
      m1 = m2;
      rs1 = rs2;
      have1 = have2;
    } else {
#pragma unroll
      for (int r = 0; r < R; r++) cur[r] = nxt[r];
      g = g2;
      m = m2;
      rs = rs2;
      have = have2;
    }
  }
}

// x for token `tok` into xs in layout LAYOUT (0 padded, 1 + QT packed
// pairs), RMSNorm-ed when a.norm_gain is set; `from` (if given) replaces
// a.x + tok * x_stride as the source row.  The caller synchronises the block
// afterwards.
template <int LAYOUT = 0>
FLOCK_DEV void gemv_stage_x(const GemvArgs& a, int tok, float* xs, float* gs, float* red,
                            const float* from = nullptr) {
  const float* x = from ? from : a.x + (size_t)tok * a.x_stride;
  if (a.norm_gain) {
    rmsnorm_to_smem<LAYOUT>(x, a.norm_gain, a.K, a.eps, xs, gs, red);
  } else if (LAYOUT != 0) {
    stage_x_packed<LAYOUT - 1>(x, a.K, xs, threadIdx.x, GEMV_THREADS);
  } else {
    const float4* src = reinterpret_cast<const float4*>(x);
#pragma unroll 4
    for (int i = threadIdx.x; i < a.K / 4; i += GEMV_THREADS)
      reinterpret_cast<float4*>(xs)[(i >> 3) * (XPAD / 4) + (i & 7)] = src[i];
  }
}

// EPI_ARGMAX: CTA reduction of the per-warp bests, then the last CTA to
// arrive reduces the per-CTA partials (kernels/argmax.wgsl pass1/pass2
// fused) into *am_best_val / *am_best_idx and re-arms the counter.  Returns
// true in every thread of that last CTA.
FLOCK_DEV bool gemv_argmax_finish(const GemvArgs& a, float best_v, uint32_t best_i,
                                  float* cta_val, uint32_t* cta_idx) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    cta_val[warp] = best_v;
    cta_idx[warp] = best_i;
  }
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    float bv = cta_val[0];
    uint32_t bi = cta_idx[0];
    for (int w = 1; w < GEMV_WARPS; w++)
      if (am_better(cta_val[w], cta_idx[w], bv, bi)) {
        bv = cta_val[w];
        bi = cta_idx[w];
      }
    a.am_val[blockIdx.x] = bv;
    a.am_idx[blockIdx.x] = bi;
    __threadfence();
    const uint32_t prev = atomicAdd(a.am_count, 1u);
    last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (last) {
    __threadfence();
    float bv = -FLT_MAX;
    uint32_t bi = 0xFFFFFFFFu;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += GEMV_THREADS) {
      const float v = ((volatile float*)a.am_val)[i];
      const uint32_t ix = ((volatile uint32_t*)a.am_idx)[i];
      if (am_better(v, ix, bv, bi)) {
        bv = v;
        bi = ix;
      }
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, bv, s);
      const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, s);
      if (am_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      cta_val[warp] = bv;
      cta_idx[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      bv = cta_val[0];
      bi = cta_idx[0];
      for (int w = 1; w < GEMV_WARPS; w++)
        if (am_better(cta_val[w], cta_idx[w], bv, bi)) {
          bv = cta_val[w];
          bi = cta_idx[w];
        }
      *a.am_best_val = bv;
      *a.am_best_idx = (int32_t)bi;
      *a.am_count = 0;  // re-arm for the next launch
    }
  }
  return last;
}

// MINB: resident CTAs per SM the register budget is sized for.
template <int QT, int R, int EPI, int MX, int LA = 1, int MINB = 2, int PK = 0>
__global__ void __launch_bounds__(GEMV_THREADS, MINB) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(16) float smem[];
  const bool norm = a.norm_gain != nullptr;
  const int kpad = a.K / 32 * XPAD;
  float* xs = smem;                          // [K/32][36] the (normalised) input
  float* gs = smem + kpad;                   // [K] gain staging (norm only)
  float* red = gs + (norm ? a.K : 0);        // [136] reduction scratch
  float* cta_val = red + 136;                // [GEMV_WARPS]
  uint32_t* cta_idx = (uint32_t*)(cta_val + GEMV_WARPS);
  float best_v = -FLT_MAX;
  uint32_t best_i = 0xFFFFFFFFu;
  // weights do not depend on any earlier kernel: their first loads go out
  // before griddepcontrol.wait, overlapping the previous kernel's tail
  gemv_run<QT, R, EPI, MX, LA, PK>(a, blockIdx.y, blockIdx.x, gridDim.x, xs, [&] {
    issue_prefetch(a.pf);
    pdl_launch_dependents();
    pdl_wait();
    if (a.ctl && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
      a.ctl[0] += a.ctl[1];
      a.ctl[1] = a.ctl_n;
    }
    gemv_stage_x<PK ? 1 + QT : 0>(a, blockIdx.y, xs, gs, red);
    __syncthreads();
  }, best_v, best_i);
  if (EPI == EPI_ARGMAX) gemv_argmax_finish(a, best_v, best_i, cta_val, cta_idx);
}

// Shared-memory bytes a k_gemv launch needs.
inline size_t gemv_smem_bytes(int K, bool norm) {
  return (size_t)(K / 32 * XPAD + (norm ? K : 0) + 136 + GEMV_WARPS * 2) * 4 + 16;
}

// Rows of two or three column blocks per lane (K = 2048, 3072: the 0.6B
// o_proj and down), one row per warp PAIR: warp 2p folds the row's even
// column steps (logical lanes 0..31 of the coop(64) order), warp 2p + 1 its
// odd steps (logical lanes 32..63), each into its own accumulator in step
// order as gemv_run does; the odd warp hands its 32 partials over through
// shared memory and the even warp adds them lane by lane -- the tree's
// first level, fadd(accA, accB) -- then finishes the tree and the epilogue.
// The same arithmetic as gemv_run; every weight load of a warp goes out
// before the dependency wait, and each warp folds half the row.
constexpr int GEMV_PAIRS = GEMV_WARPS / 2;
template <int QT, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS, 2) k_gemv_pair(const GemvArgs a) {
  extern __shared__ __align__(16) float smem[];
  const bool norm = a.norm_gain != nullptr;
  const int kpad = a.K / 32 * XPAD;
  float* xs = smem;
  float* gs = smem + kpad;
  float* red = gs + (norm ? a.K : 0);
  float* pbuf = red + 136;  // [GEMV_PAIRS][32] the odd warps' partials
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int half = warp & 1;
  const int row = blockIdx.x * GEMV_PAIRS + (warp >> 1);
  const int tok = blockIdx.y;
  const GemvSeg& sg = a.seg[0];
  const int nb = a.K / 32;
  const int M = (nb + 31) / 32;  // 2 or 3
  const bool ok = row < sg.rows;
  // this warp's steps m = half, half + 2 (< M): weights only, before the wait
  BlockW<QT> w[2];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int m = half + 2 * i, b = lane + 32 * m;
    if (ok && m < M && b < nb) load_block<QT>(w[i], sg, row, b, a.K);
  }
  issue_prefetch(a.pf);
  pdl_launch_dependents();
  pdl_wait();
  if (a.ctl && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
    a.ctl[0] += a.ctl[1];
    a.ctl[1] = a.ctl_n;
  }
  float resv = 0.0f;
  if (EPI == EPI_RESIDUAL && ok && half == 0 && lane == 0)
    resv = a.res[(size_t)tok * a.res_stride + row];
  gemv_stage_x<0>(a, tok, xs, gs, red);
  __syncthreads();
  const float4* xs4 = reinterpret_cast<const float4*>(xs);
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int m = half + 2 * i, b = lane + 32 * m;
    if (ok && m < M && b < nb) acc = fold_block<QT>(w[i], xs4 + b * (XPAD / 4), acc);
  }
  if (half == 1) pbuf[(warp >> 1) * 32 + lane] = acc;
  __syncthreads();
  if (half == 0 && ok) {
    const float y = warp_tree_sum(fadd(acc, pbuf[(warp >> 1) * 32 + lane]));
    if (lane == 0) {
      float v = y;
      if (EPI == EPI_RESIDUAL) v = fadd(resv, v);
      sg.out[(size_t)tok * sg.out_stride + row] = v;
    }
  }
}

inline size_t gemv_pair_smem_bytes(int K, bool norm) {
  return (size_t)(K / 32 * XPAD + (norm ? K : 0) + 136 + GEMV_PAIRS * 32) * 4 + 16;
}

}  // namespace flock
