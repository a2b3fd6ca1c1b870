// Fused decode FFN: ffn_norm -> gate/up -> SwiGLU -> down -> + residual in
// ONE kernel, for shapes whose gate/up rows are one 32-weight block per lane
// (hidden <= 1024) -- the 0.6B decode step, where every kernel boundary costs
// more than the work inside it.
//
// The split follows the reference's coop(64) order of the down matvec
// (kernels/q8_coop.wgsl:76): logical lane l of a down row folds the row's
// blocks l, l + 64, l + 128, ... in order and the 64 lane sums meet in the
// pairwise tree.  Block b of down's input is act[32b .. 32b + 32), which only
// needs gate/up rows 32b .. 32b + 31.  So CTA l (one per logical lane):
//   1. RMSNorm(h) * ffn_norm into shared memory (rmsnorm_to_smem);
//   2. the act blocks it owns: gate and up rows 32b .. 32b + 31 for
//      b = l, l + 64, ..., each a coop(64) row dot (one block per lane, the
//      tree), then SwiGLU -- k_gemv<.., EPI_SWIGLU>'s arithmetic;
//   3. its lane partial of every down row, P_l[r] (fold_block over its blocks
//      in order, as k_gemv's accA / accB chains), into global memory;
//   4. a grid barrier over the 64 CTAs (all resident: 64 <= SMs; bounded by
//      the global timer, a timeout sets the error word), then CTA c folds
//      rows 16c .. 16c + 15: y = tree(P_t + P_{t+32}) and h[r] += y.
// Every step is the unfused path's arithmetic in its order, so h is the
// same to the bit.  The dependent kernel is released only after the
// barrier, so no later kernel can hold an SM this grid still needs.
#pragma once
#include "common.cuh"
#include "gemv.cuh"
#include "mbar.cuh"

namespace flock {

constexpr int FFN_CTAS = 64;  // the coop(64) logical lanes
constexpr int FFN_THREADS = 256;

struct FfnArgs {
  const uint8_t* gate_qs;
  const uint16_t* gate_sc;
  const uint8_t* up_qs;
  const uint16_t* up_sc;
  const uint8_t* down_qs;
  const uint16_t* down_sc;
  int gu_sc_stride, down_sc_stride;
  int H, F;
  const float* ffn_norm;
  float eps;
  float* h;         // [H], read (norm input, residual) and written
  float* part;      // [64][H] lane partials
  unsigned long long* ticket;  // arrival counter, never reset
  int* err;         // 4 = the barrier timed out
  PrefetchList pf;  // next kernel's weights
};

// Shared memory: x padded [H/32][36] | gain [H] | red [136] | act [F].
inline size_t ffn_smem_bytes(int H, int F) {
  return (size_t)(H / 32 * XPAD + H + 136 + F) * 4 + 16;
}

// Kernel shape rule: gate/up rows of one block per lane, and each logical
// lane owning at most FFN_MAX_OWN act blocks.
constexpr int FFN_MAX_OWN = 4;
inline bool ffn_fused_fits(int H, int F) {
  return H % 32 == 0 && H <= 1024 && F % 32 == 0 && F / 32 <= FFN_CTAS * FFN_MAX_OWN;
}

static __global__ void __launch_bounds__(FFN_THREADS) k_ffn_fused(const FfnArgs a) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;
  float* gs = xs + a.H / 32 * XPAD;
  float* red = gs + a.H;
  float* act = red + 136;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int l = blockIdx.x;
  const int nbH = a.H / 32, nbF = a.F / 32;

  pdl_wait();
  // 1. x = RMSNorm(h) * ffn_norm (k_gemv's fused prologue)
  rmsnorm_to_smem(a.h, a.ffn_norm, a.H, a.eps, xs, gs, red);
  __syncthreads();
  float4 xr[8];
#pragma unroll
  for (int j = 0; j < 8; j++)
    xr[j] = lane < nbH ? reinterpret_cast<const float4*>(xs)[lane * (XPAD / 4) + j]
                       : make_float4(0.f, 0.f, 0.f, 0.f);

  // 2. act blocks b = l + 64k: warp w takes row pairs (gate, up) 4w .. 4w+3
  //    of each block; one row dot = lane folds block `lane`, then the tree
  for (int b = l; b < nbF; b += FFN_CTAS) {
    const int r0 = 32 * b + 4 * warp;
    BlockW<QT_Q8> wg[4], wu[4];
    if (lane < nbH) {
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const size_t row = (size_t)(r0 + k);
        const uint8_t* pg = a.gate_qs + row * a.H + (size_t)lane * 32;
        const uint8_t* pu = a.up_qs + row * a.H + (size_t)lane * 32;
        wg[k].w0 = ldg_stream(pg);
        wg[k].w1 = ldg_stream(pg + 16);
        wg[k].s = __ldg(a.gate_sc + row * a.gu_sc_stride + lane);
        wu[k].w0 = ldg_stream(pu);
        wu[k].w1 = ldg_stream(pu + 16);
        wu[k].s = __ldg(a.up_sc + row * a.gu_sc_stride + lane);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
      float ag = 0.0f, au = 0.0f;
      if (lane < nbH) {
        ag = fold_block<QT_Q8>(wg[k], xr, 0.0f);
        au = fold_block<QT_Q8>(wu[k], xr, 0.0f);
      }
      // k_gemv: y = tree(accA + accB) with accB = 0 for one-block rows
      const float gt = warp_tree_sum(fadd(ag, 0.0f));
      const float up = warp_tree_sum(fadd(au, 0.0f));
      if (lane == 0) {
        // ops_ref.ts:103 swigluRef: fr(fr(g / fr(1 + fr(exp(-g)))) * up)
        const float e = exp_f64r(-gt);
        act[32 * b + 4 * warp + k] = fmul(fdiv(gt, fadd(1.0f, e)), up);
      }
    }
  }
  __syncthreads();

  // 3. this lane's partial of every down row: blocks l, l + 64, ... in order
  for (int r = t; r < a.H; r += FFN_THREADS) {
    float acc = 0.0f;
    for (int b = l; b < nbF; b += FFN_CTAS) {
      BlockW<QT_Q8> w;
      const uint8_t* p = a.down_qs + (size_t)r * a.F + (size_t)b * 32;
      w.w0 = ldg_stream(p);
      w.w1 = ldg_stream(p + 16);
      w.s = __ldg(a.down_sc + (size_t)r * a.down_sc_stride + b);
      acc = fold_block<QT_Q8>(w, reinterpret_cast<const float4*>(act + 32 * b), acc);
    }
    a.part[(size_t)l * a.H + r] = acc;
  }

  // 4. grid barrier over the 64 CTAs (a ticket counter that only grows)
  __threadfence();
  __syncthreads();
  __shared__ int s_ok;
  if (t == 0) {
    const unsigned long long mine = atomicAdd(a.ticket, 1ull);
    const unsigned long long target = (mine / FFN_CTAS + 1) * FFN_CTAS;
    int ok = 1;
    uint64_t t0 = 0;
    for (uint32_t i = 0; *(volatile unsigned long long*)a.ticket < target; i++) {
      if ((i & 31) != 31) continue;
      const uint64_t now = globaltimer_ns();
      if (!t0) t0 = now;
      if (now - t0 > WAIT_NS || i >= WAIT_MAX_POLLS) {
        atomicExch(a.err, 4);
        ok = 0;
        break;
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  issue_prefetch(a.pf);
  pdl_launch_dependents();
  __threadfence();
  // the 64-lane tree of rows 16l .. 16l + 15 (k_gemv: tree(accA + accB),
  // accA = logical lane t, accB = logical lane t + 32), then + residual
  const int rows_per = (a.H + FFN_CTAS - 1) / FFN_CTAS;
  for (int k = warp; k < rows_per; k += FFN_THREADS / 32) {
    const int r = l * rows_per + k;
    if (r >= a.H) break;
    const float pa = __ldcg(a.part + (size_t)lane * a.H + r);
    const float pb = __ldcg(a.part + (size_t)(lane + 32) * a.H + r);
    const float y = warp_tree_sum(fadd(pa, pb));
    if (lane == 0) a.h[r] = fadd(a.h[r], y);
  }
}

}  // namespace flock
