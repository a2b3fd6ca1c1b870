// Reassociated Q8_0 / Q4_0 matvec for one token on the int8 tensor cores
// (FLOCK_MATVEC_FAST; the exact-order k_gemv is the default).
//
// Same function as kernels/q8_coop.wgsl:76 / q4_coop.wgsl:48 (y = W x with
// per-32-weight f16 scales), but not in the reference's f32 order: the
// parity bar is a relative error (1e-3 by contract, ~1e-6 measured), not
// bit equality.  The exact order costs about three instructions per weight
// (int8 -> f32 decode, product chains, the pairwise tree); here the weights
// go into mma.sync m16n8k32 s8 x s8 -> s32 as loaded, with no per-weight
// instruction, and only the per-block scaling runs on the SIMT pipes.
// Measured on the 151936 x 1024 head it is not faster: 43 us against the
// exact kernel's 36 (ncu: 21.5 M warp instructions against 26.8 M, about 70
// per MMA -- the per-(row, block) scaling, its loads and conversions -- and
// the exact kernel issue-bound at 66 % issue activity, this one waiting on
// its loads -- long scoreboard the top stall -- at 51 %; an L2 bulk prefetch
// of the group after next did not change it), so the exact kernel stays the
// default and this one an option.
//
// x as exact integers: per 32-element block b, with sx = max |x| and
// inv = 127 / sx, r = x * inv is split into three int8 digits
//   d0 = rint(r), d1 = rint((r - d0) * 254), d2 = rint(((r - d0) * 254 - d1) * 254)
// (each in [-127, 127]), so x = (d0 + d1 / 254 + d2 / 254^2) / inv to within
// 0.5 / 254^2 of the block maximum (~6e-8 relative).  One MMA of 16 weight
// rows x 32 columns (one block) x the 3 digit columns gives exact int32 dot
// products D_j; the row's block sum is  w_b * sum_j D_j * ws_j  with ws_j =
// 1 / (inv * 254^j) and w_b the row's f16 block scale.
//
// Fragments (PTX ISA m16n8k32 .s8, lane = 4 g + t):
//   A (weights, 16 x 32): a0 / a2 = row g, a1 / a3 = row g + 8; Q8_0 lane t
//     loads bytes 8t .. 8t+7 of the row's block (one 64-bit load) -- MMA
//     column slots 4t.. and 16+4t.. hold block columns 8t.. and 8t+4..; Q4_0
//     lane t loads nibble bytes 4t .. 4t+3 -- low nibbles are columns 4t..,
//     high nibbles 16+4t.. (the slots themselves), taken as 0..15 with
//     8 * sum_k d_j (per block and digit) subtracted from D afterwards;
//   B (digits, 32 x 8): column n = g holds digit g (g < 3; zero otherwise),
//     laid out in shared memory in the A fragment's column order;
//   D: c0 / c1 = row g, digits 2t / 2t+1; c2 / c3 = row g + 8 -- lanes t = 0
//     (digits 0, 1) and t = 1 (digit 2) carry the sums, the quad adds them.
// A warp owns 16 rows and walks the blocks in chunks of GF_CHUNK, the next
// chunk's weight and scale loads in flight while one is folded.
#pragma once
#include "gemv.cuh"

namespace flock {

constexpr int GF_ROWS = 16;   // rows per warp step (the MMA's M)
constexpr int GF_CHUNK = 4;   // blocks per chunk of loads in flight

// One chunk of a warp's loads: weights of rows g and g + 8 for GF_CHUNK
// blocks, and the rows' f16 scales of those blocks.
template <int QT>
struct GfChunk {
  uint2 w0[GF_CHUNK], w1[GF_CHUNK];  // Q4_0: .x only
  uint2 s0, s1;                      // GF_CHUNK f16 scales of each row
};

// A chunk's loads for the rows at p0 / p8 (this lane's first byte of block 0
// of rows g and g + 8; null past the segment's last row).  FULL: all
// GF_CHUNK blocks exist (no per-block guard).
template <int QT, bool FULL>
FLOCK_DEV void gf_load(GfChunk<QT>& c, const uint8_t* p0, const uint8_t* p8, const uint16_t* s0,
                       const uint16_t* s8, int b0, int nb) {
  constexpr int BB = QT == QT_Q8 ? 32 : 16;  // bytes per row block
#pragma unroll
  for (int j = 0; j < GF_CHUNK; j++) {
    const bool ok = FULL || b0 + j < nb;
    if (QT == QT_Q8) {
      c.w0[j] = (ok && p0) ? __ldg(reinterpret_cast<const uint2*>(p0 + (b0 + j) * BB)) : make_uint2(0u, 0u);
      c.w1[j] = (ok && p8) ? __ldg(reinterpret_cast<const uint2*>(p8 + (b0 + j) * BB)) : make_uint2(0u, 0u);
    } else {
      c.w0[j].x = (ok && p0) ? __ldg(reinterpret_cast<const uint32_t*>(p0 + (b0 + j) * BB)) : 0u;
      c.w1[j].x = (ok && p8) ? __ldg(reinterpret_cast<const uint32_t*>(p8 + (b0 + j) * BB)) : 0u;
    }
  }
  // the scale rows are padded to a multiple of 8 blocks: 8 aligned bytes
  c.s0 = p0 ? __ldg(reinterpret_cast<const uint2*>(s0 + b0)) : make_uint2(0u, 0u);
  c.s1 = p8 ? __ldg(reinterpret_cast<const uint2*>(s8 + b0)) : make_uint2(0u, 0u);
}

FLOCK_DEV void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                      uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Two f16 scales in a word -> f32 (scale_f16's values: e == 31 clamps to the
// largest finite f32 of its sign).
FLOCK_DEV float2 scale_f16x2(uint32_t w) {
  float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
  if ((w & 0x7C00u) == 0x7C00u) f.x = (w & 0x8000u) ? -FLT_MAX : FLT_MAX;
  if ((w & 0x7C000000u) == 0x7C000000u) f.y = (w & 0x80000000u) ? -FLT_MAX : FLT_MAX;
  return f;
}

// Shared memory: x staging as k_gemv (padded f32 + gain + reduction
// scratch), the digit image [nb][3][32] int8, ws [nb][8] f32 (digit weights,
// columns 3..7 zero), the Q4_0 digit sums [nb][8] int32 (8 * sum_k d_j).
inline size_t gemv_fast_smem_bytes(int K, bool norm) {
  const int nb = K / 32;
  return gemv_smem_bytes(K, norm) + (size_t)nb * 96 + (size_t)nb * 32 * 2 + 16;
}

template <int QT, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS, 2) k_gemv_fast(const GemvArgs a) {
  extern __shared__ __align__(16) float smem[];
  const bool norm = a.norm_gain != nullptr;
  const int nb = a.K / 32;
  const int kpad = nb * XPAD;
  float* xs = smem;
  float* gs = smem + kpad;
  float* red = gs + (norm ? a.K : 0);
  float* cta_val = red + 136;
  uint32_t* cta_idx = (uint32_t*)(cta_val + GEMV_WARPS);
  float* wsm = reinterpret_cast<float*>(cta_idx + GEMV_WARPS + 2);  // [nb][8]
  int* ssm = reinterpret_cast<int*>(wsm + nb * 8);                  // [nb][8]
  int8_t* dig = reinterpret_cast<int8_t*>(ssm + nb * 8);            // [nb][3][32]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int tok = blockIdx.y;

  int rows = 0;
  for (int s = 0; s < a.nseg; s++) rows += (a.seg[s].rows + GF_ROWS - 1) / GF_ROWS;
  const int n_groups = rows;  // row groups of 16 over all segments
  const int nwarps = gridDim.x * GEMV_WARPS;
  auto group_rows = [&](int grp, int& seg, int& row0) {
    seg = 0;
    for (int s = 0; s < a.nseg; s++) {
      const int ng = (a.seg[s].rows + GF_ROWS - 1) / GF_ROWS;
      if (grp < ng) {
        seg = s;
        row0 = grp * GF_ROWS;
        return;
      }
      grp -= ng;
    }
    row0 = 0;
  };

  // the first chunk's weights do not depend on any earlier kernel
  int grp = blockIdx.x * GEMV_WARPS + warp;
  int seg = 0, row0 = 0;
  constexpr int BB = QT == QT_Q8 ? 32 : 16;
  const int off_t = QT == QT_Q8 ? 8 * t : 4 * t;
  const uint8_t *p0 = nullptr, *p8 = nullptr;
  const uint16_t *s0 = nullptr, *s8 = nullptr;
  auto rows_at = [&](int sgi, int r0) {
    const GemvSeg& sp = a.seg[sgi];
    const size_t rb = (size_t)(a.K / 32) * BB;
    p0 = r0 + g < sp.rows ? sp.qs + (size_t)(r0 + g) * rb + off_t : nullptr;
    p8 = r0 + g + 8 < sp.rows ? sp.qs + (size_t)(r0 + g + 8) * rb + off_t : nullptr;
    s0 = sp.sc + (size_t)(r0 + g) * sp.sc_stride;
    s8 = sp.sc + (size_t)(r0 + g + 8) * sp.sc_stride;
  };
  const bool full_chunks = nb % GF_CHUNK == 0;
  GfChunk<QT> bufA, bufB;  // the current chunk and the one in flight, alternately
  if (grp < n_groups) {
    group_rows(grp, seg, row0);
    rows_at(seg, row0);
    if (full_chunks) gf_load<QT, true>(bufA, p0, p8, s0, s8, 0, nb);
    else gf_load<QT, false>(bufA, p0, p8, s0, s8, 0, nb);
  }
  issue_prefetch(a.pf);
  pdl_launch_dependents();
  pdl_wait();
  gemv_stage_x<0>(a, tok, xs, gs, red);
  __syncthreads();
  // digits: warp w takes blocks w, w + 8, ...; lane = column
  for (int b = warp; b < nb; b += GEMV_WARPS) {
    const float x = xs[b * XPAD + lane];
    float m = fabsf(x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float inv = m > 0.0f ? 127.0f / m : 0.0f;
    const float r = x * inv;
    const float d0 = rintf(r);
    const float f1 = (r - d0) * 254.0f;
    const float d1 = rintf(f1);
    const float d2 = rintf((f1 - d1) * 254.0f);
    // the A fragment's column order: Q8_0 natural, Q4_0 (4t.., 16+4t..) per lane
    const int p = QT == QT_Q8 ? lane
                              : (lane < 16 ? (lane >> 2) * 8 + (lane & 3) : ((lane - 16) >> 2) * 8 + 4 + (lane & 3));
    const int i0 = (int)d0, i1 = (int)d1, i2 = (int)d2;
    dig[(b * 3 + 0) * 32 + p] = (int8_t)i0;
    dig[(b * 3 + 1) * 32 + p] = (int8_t)i1;
    dig[(b * 3 + 2) * 32 + p] = (int8_t)i2;
    int s0 = i0, s1 = i1, s2 = i2;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (lane < 8) {
      const float w0 = m > 0.0f ? 1.0f / inv : 0.0f;
      const float w1 = w0 / 254.0f, w2 = w1 / 254.0f;
      wsm[b * 8 + lane] = lane == 0 ? w0 : lane == 1 ? w1 : lane == 2 ? w2 : 0.0f;
      ssm[b * 8 + lane] = lane == 0 ? 8 * s0 : lane == 1 ? 8 * s1 : lane == 2 ? 8 * s2 : 0;
    }
  }
  __syncthreads();

  float best_v = -FLT_MAX;
  uint32_t best_i = 0xFFFFFFFFu;
  const int n_chunks = (nb + GF_CHUNK - 1) / GF_CHUNK;
  float acc0 = 0.0f, acc1 = 0.0f;  // rows row0 + g, row0 + g + 8: this lane's digit columns
  int ci = 0;                      // chunk of the current group
  // one chunk: issue the next chunk's loads (or the next group's first)
  // into `nxt`, fold `cur`; at a group's last chunk finish its rows
  auto chunk_step = [&](const GfChunk<QT>& cur, GfChunk<QT>& nxt) {
    const GemvSeg& sg = a.seg[seg];
    const int rg = row0 + g, rg8 = row0 + g + 8;
    const bool has0 = p0 != nullptr, has8 = p8 != nullptr;
    const int b0 = ci * GF_CHUNK;
    const bool last = ci + 1 == n_chunks;
    int ngrp = grp, nseg = seg, nrow0 = row0, nb0 = b0 + GF_CHUNK;
    if (last) {
      nb0 = 0;
      ngrp = grp + nwarps;
      if (ngrp < n_groups) {
        group_rows(ngrp, nseg, nrow0);
        rows_at(nseg, nrow0);
      }
    }
    if (ngrp < n_groups) {
      if (full_chunks) gf_load<QT, true>(nxt, p0, p8, s0, s8, nb0, nb);
      else gf_load<QT, false>(nxt, p0, p8, s0, s8, nb0, nb);
    }
    float2 sc0[GF_CHUNK / 2], sc1[GF_CHUNK / 2];
    {
      const uint32_t v0[2] = {cur.s0.x, cur.s0.y};
      const uint32_t v1[2] = {cur.s1.x, cur.s1.y};
#pragma unroll
      for (int q = 0; q < GF_CHUNK / 2; q++) {
        sc0[q] = scale_f16x2(v0[q]);
        sc1[q] = scale_f16x2(v1[q]);
      }
    }
#pragma unroll
    for (int j = 0; j < GF_CHUNK; j++) {
      const int b = b0 + j;
      if (full_chunks || b < nb) {
        uint32_t bd0 = 0u, bd1 = 0u;
        if (g < 3) {
          const uint2 v = *reinterpret_cast<const uint2*>(dig + (b * 3 + g) * 32 + 8 * t);
          bd0 = v.x;
          bd1 = v.y;
        }
        uint32_t a0, a1, a2, a3;
        if (QT == QT_Q8) {
          a0 = cur.w0[j].x;
          a2 = cur.w0[j].y;
          a1 = cur.w1[j].x;
          a3 = cur.w1[j].y;
        } else {
          a0 = cur.w0[j].x & 0x0F0F0F0Fu;
          a2 = (cur.w0[j].x >> 4) & 0x0F0F0F0Fu;
          a1 = cur.w1[j].x & 0x0F0F0F0Fu;
          a3 = (cur.w1[j].x >> 4) & 0x0F0F0F0Fu;
        }
        int d[4];
        mma_s8(d, a0, a1, a2, a3, bd0, bd1);
        if (QT == QT_Q4) {
          const int2 sv = *reinterpret_cast<const int2*>(ssm + b * 8 + 2 * t);
          d[0] -= sv.x;
          d[1] -= sv.y;
          d[2] -= sv.x;
          d[3] -= sv.y;
        }
        const float2 ws = *reinterpret_cast<const float2*>(wsm + b * 8 + 2 * t);
        const float v0 = fmaf((float)d[1], ws.y, (float)d[0] * ws.x);
        const float v1 = fmaf((float)d[3], ws.y, (float)d[2] * ws.x);
        acc0 = fmaf(v0, (j & 1) ? sc0[j >> 1].y : sc0[j >> 1].x, acc0);
        acc1 = fmaf(v1, (j & 1) ? sc1[j >> 1].y : sc1[j >> 1].x, acc1);
      }
    }
    ci++;
    if (!last) return;
    // end of this group: the quad's lanes hold digit columns 2t, 2t+1
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    if (t == 0) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int r = h ? rg8 : rg;
        if (!(h ? has8 : has0)) continue;
        float v = h ? acc1 : acc0;
        if (EPI == EPI_RESIDUAL) v = v + a.res[(size_t)tok * a.res_stride + r];
        sg.out[(size_t)tok * sg.out_stride + r] = v;
        if (EPI == EPI_ARGMAX) {
          const uint32_t idx = (uint32_t)(r + a.am_row_offset);
          if (am_better(v, idx, best_v, best_i)) {
            best_v = v;
            best_i = idx;
          }
        }
      }
    }
    acc0 = acc1 = 0.0f;
    ci = 0;
    grp = ngrp;
    seg = nseg;
    row0 = nrow0;
  };
  while (grp < n_groups) {
    chunk_step(bufA, bufB);
    if (grp >= n_groups) break;
    chunk_step(bufB, bufA);
  }
  if (EPI == EPI_ARGMAX) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, best_v, o);
      const uint32_t oi = __shfl_down_sync(0xffffffffu, best_i, o);
      if (am_better(ov, oi, best_v, best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    gemv_argmax_finish(a, best_v, best_i, cta_val, cta_idx);
  }
}

}  // namespace flock
