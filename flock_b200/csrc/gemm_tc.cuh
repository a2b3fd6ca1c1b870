// Prefill GEMM on the 5th-generation tensor cores (tcgen05) for Q8_0 / Q4_0
// weights -- kernels/q8_coop.wgsl:76 / q4_coop.wgsl:48 at M > 1 tokens
// (layer.ts:685 encodePrefill), re-designed for B200:
//
//   Y[m][n] = sum_k X[m][k] * W[n][k],  X f32 -> f16 (a power-of-two scale
//   per token row), W = s * q -> f16, f32 accumulation in tensor memory.
//
//  * 16-bit operands are f16, not bf16: kind::f16 runs both at the same rate
//    and f16's 11-bit significand rounds 8x more finely (per-GEMM error
//    ~3e-4 instead of ~2e-3 at K = 4096-12288).  Each activation row is
//    scaled by 2^-e so its largest magnitude lies in [2^13, 2^14) before the
//    rounding (no overflow, full precision), and the epilogue multiplies by
//    2^e, which is exact.  Weights q * s are exact in f32 and rounded once.
//
//  * Operands are swapped for small M: 128 weight rows form the MMA's M and
//    up to 256 tokens its N, so a 16-token prefill still issues full-height
//    tcgen05.mma.cta_group::1.kind::f16 (128 x Nt x 16) instructions.
//  * Raw weight tiles arrive by TMA: one thread of a loader warp issues a
//    2-D cp.async.bulk.tensor per K-tile (128 rows x 64 int8 bytes, or x 32
//    nibble bytes) from the weight's tensor map into a ring of 4
//    shared-memory stages (the map's 64-/32-byte swizzle spreads the rows
//    over all banks), completing on the stage's mbarrier by transaction
//    count.  The map always describes this GPU's own weight plane; there is
//    no multicast.  The kernel is launched with programmatic dependent
//    launch: these weight loads may start while the previous kernel (the
//    activation image) still runs; everything that kernel writes is read
//    after griddepcontrol.wait.
//  * Converters (8 warps, two threads per weight row: one 32-weight block
//    each per K-tile) read their block from the raw stage, release it,
//    form q * s in packed f16 arithmetic (exact integers, one correctly
//    rounded multiply by the stored f16 scale; the scales come from global
//    memory a few K-tiles ahead) and write the K-major
//    128-byte-swizzled layout the UMMA shared-memory descriptor names
//    (8-row x 128-byte atoms, 16-byte chunk c of row r at (c ^ r % 8)).  The
//    only weight rounding is that of the scaled value.
//  * Activations come from an image the caller builds once per GEMM
//    (k_act_image: RMSNorm fused, f16, same swizzled layout, Nt rows per
//    K-tile contiguous), so each stage's B tile is one bulk copy.
//  * One thread issues the MMAs; tcgen05.commit returns each stage to the
//    converters through an mbarrier and signals the epilogue after the last
//    K-tile.  The 8 converter warps then read the accumulator with tcgen05.ld
//    (32 lanes x 32 bit: one weight row per thread, one token per column;
//    warps w and w+4 share a lane quarter and split the columns) and store
//    coalesced rows of Y, optionally adding a residual.
//
// Every wait is bounded (mbar_wait); on a timeout the kernel sets *err,
// still releases its tensor memory and returns.  No multicast is used.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "gemv.cuh"
#include "mbar.cuh"

namespace flock {

constexpr int TC_ROWS = 128;              // weight rows per CTA: the MMA's M
constexpr int TC_KT = 64;                 // K per stage: one 128-byte f16 swizzle atom row
constexpr int TC_STAGES = 4;              // f16 A / image B stages
constexpr int TC_RAW_MAX = 12;            // raw weight stages (TMA ring), at most
constexpr int TC_SMEM_MAX = 232448;       // dynamic shared memory per CTA on sm_100
constexpr int TC_MAX_NT = 256;            // tokens per CTA: the MMA's N
constexpr int TC_PRODUCERS = 256;         // 8 warps: converters, then the epilogue
constexpr int TC_THREADS = TC_PRODUCERS + 96;  // + the MMA warp + the weight and image loaders
constexpr int TC_A_BYTES = TC_ROWS * TC_KT * 2;  // 16 KiB of f16 per stage
constexpr int TC_RAW_BYTES = TC_ROWS * TC_KT;    // 8 KiB of int8 per raw stage (Q4: half used)
constexpr int TC_SC_AHEAD = 4;            // K-tiles of scales loaded ahead per thread

struct TcSeg {
  const uint8_t* qs;
  const uint16_t* sc;
  int sc_stride;   // f16 scales per row
  int rows;
  float* out;      // [m][out_stride]
  int out_stride;
};

struct TcArgs {
  // 2-D tensor map of each segment's qs plane: {row bytes, rows}, box
  // {64 (Q8) / 32 (Q4) bytes, 128 rows}, 64-/32-byte swizzle (host-encoded)
  CUtensorMap tmap[3];
  TcSeg seg[3];
  int nseg;
  int tile0[4];      // first 128-row tile of each segment; tile0[nseg] = all tiles
  int K, M, Nt;      // Nt: tokens per CTA (multiple of 16, <= 256)
  int img_nt;        // token rows per image tile (Nt divides it)
  const uint8_t* img;  // activation image: [M / img_nt][K / 64][img_nt][128 B] f16, swizzled
  const int* row_exp;  // e of each image row: the row was scaled by 2^-e
  const float* res;    // EPI_RESIDUAL: y += res[m][n] (res may alias the output)
  int res_stride;
  int* err;
  // split-K (one segment): CTA z covers K-tiles [z * KT / ksplit, (z+1) * KT / ksplit)
  // and writes its partial to part[z][m][row]; k_splitk_reduce sums them
  int ksplit;
  float* part;
  int raw_stages;    // depth of the raw weight ring (tc_raw_stages)
};

// ------------------------------------------------------------------ tcgen05
FLOCK_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FLOCK_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
FLOCK_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
FLOCK_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
FLOCK_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D[tmem] (+)= A[smem desc] . B[smem desc]^T, f16 inputs, f32 accumulator.
FLOCK_DEV void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The mbarrier arrives once every tcgen05 operation this thread issued before
// has completed.
FLOCK_DEV void umma_commit(uint64_t* mbar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(mbar))
      : "memory");
}
// 16 consecutive f32 columns of this warp's 32 tensor-memory lanes.
FLOCK_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 bytes apart (stride byte offset); the leading byte offset is unused
// for swizzled K-major operands.  Bits 46-47 hold the sm_100 descriptor
// version (1), bits 61-63 the layout (2 = 128-byte swizzle).
FLOCK_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: f32 D (bits 4-5 = 1), f16 A and B
// (bits 7-9, 10-12 = 0), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
FLOCK_DEV uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Byte offset of 16-byte chunk c (8 f16, K elements 8c..8c+7 of a K-tile)
// of row r inside a K-tile block of 128-byte rows.
FLOCK_DEV uint32_t sw128_off(int r, int c) { return (uint32_t)r * 128u + (uint32_t)((c ^ (r & 7)) << 4); }

// Two f32 -> f16 (round to nearest even), lo in the low half.
FLOCK_DEV uint32_t h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// e with max_abs in [2^(e+13), 2^(e+14)): scaling a row by 2^-e puts its
// largest magnitude in [2^13, 2^14).  0 for an all-zero row; clamped to
// [-120, 120] so 2^e and 2^-e are normal floats.
FLOCK_DEV int row_exponent(float max_abs) {
  const int biased = (int)((__float_as_uint(max_abs) >> 23) & 0xFFu);
  const int e = biased == 0 ? 0 : biased - 127 - 13;
  return e < -120 ? -120 : (e > 120 ? 120 : e);
}
// 2^e for e in [-126, 127], exactly.
FLOCK_DEV float pow2f(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// Raw weights of one block (32 weights) of a row for one K-tile.
struct TcRaw {
  uint4 q[2];   // Q8: 32 int8; Q4: q[0] = the 16-byte nibble block
  uint32_t s;   // the f16 scale (low 16 bits)
};

// Block `half` (0/1) of row t from a raw stage the TMA wrote.  Q8 rows are
// 64 bytes with the 64-byte swizzle (16-byte chunk c of row t at
// c ^ ((t >> 1) & 3)); Q4 rows are 32 bytes with the 32-byte swizzle (chunk
// c at c ^ ((t >> 2) & 1)).  Either way the 8 threads of an LDS.128 phase
// (four rows, both halves) hit 8 distinct 4-bank groups.
template <int QT>
FLOCK_DEV void tc_read_raw(TcRaw& r, const uint8_t* raw, int t, int half) {
  if (QT == QT_Q8) {
    const int x = (t >> 1) & 3;
    const uint8_t* row = raw + t * 64;
    r.q[0] = *reinterpret_cast<const uint4*>(row + (((2 * half) ^ x) << 4));
    r.q[1] = *reinterpret_cast<const uint4*>(row + (((2 * half + 1) ^ x) << 4));
  } else {
    r.q[0] = *reinterpret_cast<const uint4*>(raw + t * 32 + ((half ^ ((t >> 2) & 1)) << 4));
  }
}

// 2-D tiled TMA load of box {x, y} into shared memory, completing on `bar`
// by transaction bytes.  `tmap` is the generic address of a tensor map in
// kernel parameter space (__grid_constant__).
FLOCK_DEV void tma_load_2d(void* dst, const CUtensorMap* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
FLOCK_DEV void tma_prefetch_desc(const CUtensorMap* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// f16(q * s) for the four 8-bit values of word u (bytes v = q + bias, v in
// [0, 255]), two per packed f16 op: __byte_perm places each byte under the
// exponent 0x64 (f16 1024 + v, exact), one HSUB2 removes 1024 + bias
// (exact: the values are integers below 2048) and one HMUL2 by the block's
// f16 scale rounds q * s to f16 once, to nearest even -- the same bits as
// rounding the exact f32 product.
FLOCK_DEV uint2 tc_dequant4(uint32_t u, __half2 bias2, __half2 s2) {
  const uint32_t lo = __byte_perm(u, 0x64646464u, 0x5140u);  // (v0, v1) + 1024
  const uint32_t hi = __byte_perm(u, 0x64646464u, 0x7362u);  // (v2, v3) + 1024
  const __half2 a = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&lo), bias2), s2);
  const __half2 b = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&hi), bias2), s2);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

// Dequantise one block into chunks 4*half .. 4*half+3 of row t's swizzled
// 128-byte row of the A stage: q * s rounded once to f16 (q exact, s the
// block's f16 scale as stored).
template <int QT>
FLOCK_DEV void tc_store_block(const TcRaw& r, uint8_t* A, int t, int half) {
  const uint16_t sb = (uint16_t)(r.s & 0xFFFFu);
  const __half2 s2 = __halves2half2(__ushort_as_half(sb), __ushort_as_half(sb));
  // 1024 + 128 (Q8: int8 -> u8 by flipping the sign bit) or 1024 + 8 (Q4)
  const __half2 bias2 = QT == QT_Q8 ? __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480))
                                    : __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
#pragma unroll
  for (int cc = 0; cc < 4; cc++) {
    uint32_t w0, w1;
    if (QT == QT_Q8) {
      // weights 8cc..8cc+7 of the block
      const uint4 w = r.q[cc >> 1];
      w0 = ((cc & 1) ? w.z : w.x) ^ 0x80808080u;
      w1 = ((cc & 1) ? w.w : w.y) ^ 0x80808080u;
    } else {
      // q4_coop.wgsl: byte i holds weights i (low nibble) and i+16 (high);
      // weights 8cc..8cc+7 are nibbles of bytes 8(cc&1).. , high for cc >= 2
      const uint4 w = r.q[0];
      const int sh = cc < 2 ? 0 : 4;
      w0 = (((cc & 1) ? w.z : w.x) >> sh) & 0x0F0F0F0Fu;
      w1 = (((cc & 1) ? w.w : w.y) >> sh) & 0x0F0F0F0Fu;
    }
    const uint2 lo = tc_dequant4(w0, bias2, s2), hi = tc_dequant4(w1, bias2, s2);
    *reinterpret_cast<uint4*>(A + sw128_off(t, 4 * half + cc)) = make_uint4(lo.x, lo.y, hi.x, hi.y);
  }
}

FLOCK_DEV int tc_tmem_cols(int nt) {
  int c = 32;
  while (c < nt) c <<= 1;
  return c;
}

template <int QT, int EPI>
static __global__ void __launch_bounds__(TC_THREADS, 1)
    k_gemm_tc(const __grid_constant__ TcArgs a) {
  extern __shared__ __align__(16) uint8_t tsm_raw[];
  // the swizzle atoms must sit on 1024-byte boundaries: round the dynamic
  // shared memory up (the launch reserves 1 KiB of slack for this)
  uint8_t* tsm = tsm_raw + ((1024u - (smem_u32(tsm_raw) & 1023u)) & 1023u);
  const int Nt = a.Nt;
  const int b_bytes = Nt * 128;
  const int stage_bytes = TC_A_BYTES + b_bytes;  // a multiple of 1024
  const int R = a.raw_stages;
  uint8_t* rawbase = tsm + TC_STAGES * stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(rawbase + R * TC_RAW_BYTES);
  uint64_t* bfull = full + TC_STAGES;    // the image tile's bulk copy landed
  uint64_t* empty = bfull + TC_STAGES;   // the MMAs reading the stage completed
  uint64_t* rfull = empty + TC_STAGES;   // a raw weight tile landed (TMA)
  uint64_t* rempty = rfull + TC_RAW_MAX; // every converter read its raw block
  uint64_t* done = rempty + TC_RAW_MAX;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int RAW_ROW = QT == QT_Q8 ? TC_KT : TC_KT / 2;  // raw bytes per row per K-tile
  // launched with programmatic dependent launch: this kernel reads the
  // previous kernel's output (the activation image, row scales, residual)
  // only after griddepcontrol.wait -- the weight loads before it touch
  // nothing any kernel writes
  constexpr uint32_t RAW_TX = (uint32_t)(TC_ROWS * RAW_ROW);

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; s++) {
      mbar_init(&full[s], TC_PRODUCERS);
      mbar_init(&bfull[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < R; s++) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], TC_PRODUCERS);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const uint32_t ncols = (uint32_t)tc_tmem_cols(Nt);
  if (warp == TC_PRODUCERS / 32) {
    tmem_alloc(tslot, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // every CTA holds its tensor memory: the next kernel may start its
  // prologue (and allocate tensor memory) without this grid waiting on it
  pdl_launch_dependents();

  int sgi = 0;
  while (sgi + 1 < a.nseg && (int)blockIdx.x >= a.tile0[sgi + 1]) sgi++;
  const TcSeg& sg = a.seg[sgi];
  const int row0 = ((int)blockIdx.x - a.tile0[sgi]) * TC_ROWS;
  const int mb = blockIdx.y, m0 = mb * Nt;
  const int KT = a.K / TC_KT / a.ksplit;       // K-tiles of this CTA
  const int kt_base = (int)blockIdx.z * KT;     // its first K-tile

  if (warp < TC_PRODUCERS / 32) {
    // ----------------------------------------------------------- converters
    const int t = threadIdx.x & (TC_ROWS - 1), half = threadIdx.x >> 7;
    const int row = row0 + t;
    const bool rv = row < sg.rows;
    const int lrow = rv ? row : sg.rows - 1;  // rows past the end read a real scale, store nothing
    const uint16_t* scp = sg.sc + (size_t)lrow * sg.sc_stride + half;
    uint32_t scr[TC_SC_AHEAD];
#pragma unroll
    for (int j = 0; j < TC_SC_AHEAD; j++)
      if (j < KT) scr[j] = __ldg(scp + (kt_base + j) * 2);
    bool ok = true;
    for (int kt0 = 0; kt0 < KT && ok; kt0 += TC_SC_AHEAD) {
#pragma unroll
      for (int j = 0; j < TC_SC_AHEAD; j++) {
        const int kt = kt0 + j;
        if (kt >= KT || !ok) break;
        const int st = kt % TC_STAGES, rs = kt % R;
        if (kt >= TC_STAGES &&
            !mbar_wait_poll(&empty[st], (uint32_t)(((kt / TC_STAGES) - 1) & 1), a.err)) {
          atomicCAS(a.err, 0, 1);
          ok = false;
          break;
        }
        uint8_t* A = tsm + (size_t)st * stage_bytes;
        if (!mbar_wait_poll(&rfull[rs], (uint32_t)((kt / R) & 1), a.err)) {
          atomicCAS(a.err, 0, 1);
          ok = false;
          break;
        }
        TcRaw r;
        tc_read_raw<QT>(r, rawbase + rs * TC_RAW_BYTES, t, half);
        r.s = scr[j];
        // the block is in registers: order these generic reads before the
        // loader's next (async-proxy) TMA write of the stage, then release it
        fence_proxy_async_smem();
        mbar_arrive(&rempty[rs]);
        if (kt + TC_SC_AHEAD < KT) scr[j] = __ldg(scp + (kt_base + kt + TC_SC_AHEAD) * 2);
        tc_store_block<QT>(r, A, t, half);
        fence_proxy_async_smem();
        mbar_arrive(&full[st]);
      }
    }
    // ------------------------------------------------------------- epilogue
    if (!mbar_wait(done, 0, a.err)) atomicCAS(a.err, 0, 1);
    pdl_wait();  // row scales, residual and outputs belong to the previous kernels' step
    tc_fence_after();
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const bool split = a.ksplit > 1;
    for (int c0 = 16 * half; c0 < Nt; c0 += 32) {
      // the residual (which may alias the output) is read before any store
      float r[16];
      if (EPI == EPI_RESIDUAL && !split && rv) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const int m = m0 + c0 + j;
          r[j] = m < a.M ? a.res[(size_t)m * a.res_stride + row] : 0.0f;
        }
      }
      float v[16];
      tmem_ld16(tmem + lane_base + (uint32_t)c0, v);
      if (rv) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const int m = m0 + c0 + j;
          if (m < a.M) {
            v[j] = v[j] * pow2f(a.row_exp[m]);  // undo the row's power-of-two scale (exact)
            if (split) {
              a.part[((size_t)blockIdx.z * a.M + m) * sg.rows + row] = v[j];
            } else {
              const float y = EPI == EPI_RESIDUAL ? r[j] + v[j] : v[j];
              sg.out[(size_t)m * sg.out_stride + row] = y;
            }
          }
        }
      }
    }
  } else if (warp == TC_PRODUCERS / 32) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(TC_ROWS, Nt);
      for (int kt = 0; kt < KT; kt++) {
        const int st = kt % TC_STAGES;
        const uint32_t par = (uint32_t)((kt / TC_STAGES) & 1);
        if (!mbar_wait_poll(&full[st], par, a.err) || !mbar_wait_poll(&bfull[st], par, a.err)) {
          atomicCAS(a.err, 0, 1);
          break;
        }
        tc_fence_after();
        const uint32_t A = smem_u32(tsm + (size_t)st * stage_bytes), B = A + TC_A_BYTES;
#pragma unroll
        for (int k16 = 0; k16 < TC_KT / 16; k16++)
          umma_f16(tmem, umma_desc_sw128(A + 32 * k16), umma_desc_sw128(B + 32 * k16), idesc,
                    (kt | k16) != 0);
        umma_commit(&empty[st]);
      }
      umma_commit(done);
    }
  } else if (warp == TC_PRODUCERS / 32 + 2) {
    // --------------------------------------------------------- image loader
    // the B tile of K-tile kt goes into stage kt % TC_STAGES as soon as the
    // MMAs of kt - TC_STAGES have released it
    if (lane == 0) {
      pdl_wait();  // the image is the previous kernel's output
      int issued = 0;
      bool ok = true;
      for (int kt = 0; kt < KT; kt++) {
        const int st = kt % TC_STAGES;
        if (kt >= TC_STAGES &&
            !mbar_wait_poll(&empty[st], (uint32_t)(((kt / TC_STAGES) - 1) & 1), a.err)) {
          atomicCAS(a.err, 0, 1);
          ok = false;
          break;
        }
        mbar_expect_tx(&bfull[st], (uint32_t)b_bytes);
        // this CTA's Nt rows of the image tile that holds token m0 (an Nt
        // subset of an image tile keeps the row swizzle: Nt is a multiple of 8)
        bulk_g2s(tsm + (size_t)st * stage_bytes + TC_A_BYTES,
                 a.img + ((size_t)(m0 / a.img_nt) * (a.K / TC_KT) + kt_base + kt) *
                             (size_t)a.img_nt * 128 + (size_t)(m0 % a.img_nt) * 128,
                 (uint32_t)b_bytes, &bfull[st]);
        issued = kt + 1;
      }
      if (!ok) {
        // let the copies still in flight land before the CTA can exit
        for (int kt = issued > TC_STAGES ? issued - TC_STAGES : 0; kt < issued; kt++)
          mbar_wait(&bfull[kt % TC_STAGES], (uint32_t)((kt / TC_STAGES) & 1), a.err, false);
      }
    }
  } else if (lane == 0) {
    // ----------------------------------------------------------- TMA loader
    const CUtensorMap* map = &a.tmap[sgi];
    tma_prefetch_desc(map);
    int issued = 0;
    bool ok = true;
    for (int kt = 0; kt < KT; kt++) {
      const int rs = kt % R;
      if (kt >= R && !mbar_wait_poll(&rempty[rs], (uint32_t)(((kt / R) - 1) & 1), a.err)) {
        atomicCAS(a.err, 0, 1);
        ok = false;
        break;
      }
      mbar_expect_tx(&rfull[rs], RAW_TX);
      // x: the K-tile's first byte of the row (a multiple of 32 or 64 bytes);
      // y: the tile's first row (rows past the end read as zeros)
      tma_load_2d(rawbase + rs * TC_RAW_BYTES, map, (kt_base + kt) * RAW_ROW, row0, &rfull[rs]);
      issued = kt + 1;
    }
    if (!ok) {
      // let the copies still in flight land before the CTA can exit
      for (int kt = issued > R ? issued - R : 0; kt < issued; kt++)
        mbar_wait(&rfull[kt % R], (uint32_t)((kt / R) & 1), a.err, false);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == TC_PRODUCERS / 32) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// out[m][n] = (res[m][n] +) sum_z part[z][m][n], the splits added in order.
static __global__ void k_splitk_reduce(const float* part, int ksplit, int M, int N,
                                       const float* res, int res_stride, float* out,
                                       int out_stride) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * N) return;
  const int64_t m = i / N, n = i - m * N;
  const size_t plane = (size_t)M * N;
  float p[8];  // every split's load in flight before the ordered adds
#pragma unroll
  for (int z = 0; z < 8; z++) p[z] = z < ksplit ? part[z * plane + i] : 0.0f;
  float s = p[0];
#pragma unroll
  for (int z = 1; z < 8; z++)
    if (z < ksplit) s = s + p[z];
  if (res) s = res[m * res_stride + n] + s;
  out[m * out_stride + n] = s;
}

// Shared memory besides the raw ring: A/B stages, barriers, the TMEM slot,
// and 1 KiB of alignment slack.
inline size_t gemm_tc_fixed_smem(int nt) {
  return (size_t)TC_STAGES * (TC_A_BYTES + nt * 128) + (3 * TC_STAGES + 2 * TC_RAW_MAX + 1) * 8 +
         16 + 1024;
}
// Raw weight stages (8 KiB each).  Four: a 12-stage ring (all the shared
// memory a 128-token tile leaves) measured slower on B200 -- 24.7 against
// 20.9 us for the M = 512 q/k/v GEMM -- and at M = 16 it halves the CTAs an
// SM holds.
inline int tc_raw_stages(int nt) {
  (void)nt;
  return 4;
}
inline size_t gemm_tc_smem_bytes(int nt) {
  return gemm_tc_fixed_smem(nt) + (size_t)tc_raw_stages(nt) * TC_RAW_BYTES;
}

// ------------------------------------------------------- activation image
// X (f32 [M][x_stride]) -> f16 image [M / Nt][K / 64][Nt][128 B] in the
// swizzled K-major layout, RMSNorm fused when `gain` is set (ops_ref.ts:20
// order: thread t of the row's 128 folds the strided partial t = sum over
// i = t, t+128, ... of x_i^2 with fma in order, then the pairwise tree over
// the 128 partials, 1/sqrt in f64 rounded once, then x * scale * gain rounded
// per multiply); each row is scaled by 2^-e (row_exponent of its largest
// magnitude) before rounding to f16 and e is stored in row_exp.  One CTA of
// 128 threads per image row, the row staged in shared memory; rows >= M
// are written as zeros.  The row can also be formed on the way in: merged
// from the attention's key ranges, summed from split-K partials plus the
// residual (and written back), or the SwiGLU of [gate | up].
struct ActImgArgs {
  const float* x;
  int x_stride;
  const float* gain;
  float eps;
  int M, K, Nt;
  uint8_t* img;
  int* row_exp;
  // instead of x: the key ranges of the tensor-core prefill attention
  // ([nz][M][K] unnormalised O, then [nz][M][n_heads][2] (m, l)), merged here
  const float* part;
  int nz, n_heads;
  // x = res + sum of split-K partials ([red_nz][M][K], the order of
  // k_splitk_reduce), also written back to x_out (the residual stream)
  const float* red_part;
  int red_nz;
  float* x_out;
  // x = SwiGLU of [gate | up] rows ([M][2K], ops_ref.ts:103 order)
  const float* gu;
};

constexpr int ACT_IMG_THREADS = 128;                // one CTA per row: the RMSNorm's WG
constexpr int ATC_MAX_SPLITS_IMG = 8;               // attention key ranges the merge takes

// shared memory: the row [K], the 128 partials / maxima, the merge weights
inline size_t act_image_smem_bytes(int K) {
  return ((size_t)K + ACT_IMG_THREADS + ATC_MAX_SPLITS_IMG * 32 + 32) * 4;
}

static __global__ void __launch_bounds__(ACT_IMG_THREADS) k_act_image(const ActImgArgs a) {
  extern __shared__ __align__(16) float xr[];  // [K] row, then scratch
  pdl_launch_dependents();
  // the gains are weights (no kernel writes them): this thread's float4s of
  // them, for rows of up to 4096, load before the dependency wait
  constexpr int GREG = 8;
  float4 gr[GREG];
  const bool greg = a.gain != nullptr && a.K / 4 <= GREG * ACT_IMG_THREADS;
  if (greg) {
#pragma unroll
    for (int j = 0; j < GREG; j++) {
      const int i = (int)threadIdx.x + j * ACT_IMG_THREADS;
      if (i < a.K / 4) gr[j] = __ldg(reinterpret_cast<const float4*>(a.gain) + i);
    }
  }
  pdl_wait();
  float* red = xr + a.K;                       // [128]
  float* w = red + ACT_IMG_THREADS;            // [ATC_MAX_SPLITS_IMG][32] merge weights
  float* winv = w + ATC_MAX_SPLITS_IMG * 32;   // [32]
  const int t = threadIdx.x;
  const int m = blockIdx.x;
  const int r = m % a.Nt, mb = m / a.Nt, KT = a.K / TC_KT;
  uint8_t* base = a.img + (size_t)mb * KT * a.Nt * 128;
  if (m >= a.M) {
    for (int i = t; i < a.K / 8; i += ACT_IMG_THREADS)
      *reinterpret_cast<uint4*>(base + (size_t)(i >> 3) * a.Nt * 128 + sw128_off(r, i & 7)) =
          make_uint4(0, 0, 0, 0);
    if (t == 0) a.row_exp[m] = 0;
    return;
  }
  float4* x4 = reinterpret_cast<float4*>(xr);
  const int K4 = a.K / 4;
  if (a.part) {
    // merge the attention's key ranges (k_attn_prefill_tc): thread hh derives
    // head hh's range weights e^(m_z - m) and 1 / l, l = sum_z e^(m_z - m) l_z,
    // then every element is the weighted sum of its ranges in order
    const float* ml = a.part + (size_t)a.nz * a.M * a.K;
    if (t < a.n_heads) {
      float mx = -INFINITY, l = 0.0f;
      for (int z = 0; z < a.nz; z++) {
        const float* p = ml + (((size_t)z * a.M + m) * a.n_heads + t) * 2;
        if (p[1] > 0.0f) mx = fmaxf(mx, p[0]);
      }
      for (int z = 0; z < a.nz; z++) {
        const float* p = ml + (((size_t)z * a.M + m) * a.n_heads + t) * 2;
        const float e = p[1] > 0.0f ? expf(p[0] - mx) : 0.0f;
        w[z * 32 + t] = e;
        l += e * p[1];
      }
      winv[t] = 1.0f / l;
    }
    __syncthreads();
    const int hd4 = K4 / a.n_heads;  // float4s per head
    for (int i = t; i < K4; i += ACT_IMG_THREADS) {
      const int hh = i / hd4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int z = 0; z < a.nz; z++) {
        const float wz = w[z * 32 + hh];
        if (wz != 0.0f) {
          const float4 o = reinterpret_cast<const float4*>(a.part + ((size_t)z * a.M + m) * a.K)[i];
          acc = make_float4(fmaf(wz, o.x, acc.x), fmaf(wz, o.y, acc.y), fmaf(wz, o.z, acc.z),
                            fmaf(wz, o.w, acc.w));
        }
      }
      const float inv = winv[hh];
      x4[i] = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
  } else if (a.red_part) {
    const float4* src = reinterpret_cast<const float4*>(a.x + (size_t)m * a.x_stride);
    float4* dst = reinterpret_cast<float4*>(a.x_out + (size_t)m * a.x_stride);
    const size_t plane4 = (size_t)a.M * a.K / 4;
    for (int i = t; i < K4; i += ACT_IMG_THREADS) {
      const float4* p = reinterpret_cast<const float4*>(a.red_part + (size_t)m * a.K) + i;
      float4 v = p[0];
      for (int z = 1; z < a.red_nz; z++) {
        const float4 u = p[z * plane4];
        v = make_float4(fadd(v.x, u.x), fadd(v.y, u.y), fadd(v.z, u.z), fadd(v.w, u.w));
      }
      const float4 rr = src[i];
      v = make_float4(fadd(rr.x, v.x), fadd(rr.y, v.y), fadd(rr.z, v.z), fadd(rr.w, v.w));
      x4[i] = v;
      dst[i] = v;
    }
  } else if (a.gu) {
    const float4* g4 = reinterpret_cast<const float4*>(a.gu + (size_t)m * 2 * a.K);
    const float4* u4 = reinterpret_cast<const float4*>(a.gu + (size_t)m * 2 * a.K + a.K);
    auto sw = [](float g, float u) { return fmul(fdiv(g, fadd(1.0f, exp_f64r(-g))), u); };
    for (int i = t; i < K4; i += ACT_IMG_THREADS) {
      const float4 g = g4[i], u = u4[i];
      x4[i] = make_float4(sw(g.x, u.x), sw(g.y, u.y), sw(g.z, u.z), sw(g.w, u.w));
    }
  } else {
    const float4* src = reinterpret_cast<const float4*>(a.x + (size_t)m * a.x_stride);
    for (int i = t; i < K4; i += ACT_IMG_THREADS) x4[i] = src[i];
  }
  __syncthreads();
  float scale = 1.0f;
  if (a.gain) {
    // ops_ref.ts:20: partial t over i = t, t+128, ... in order, then the tree
    // the pairwise tree: levels 64 and 32 in one step across the warps,
    // (r[l] + r[l+64]) + (r[l+32] + r[l+96]), the last five in warp 0
    float p = 0.0f;
    for (int i = t; i < a.K; i += ACT_IMG_THREADS) p = ffma(xr[i], xr[i], p);
    red[t] = p;
    __syncthreads();
    if (t < 32) {
      float v = fadd(fadd(red[t], red[t + 64]), fadd(red[t + 32], red[t + 96]));
      v = warp_tree_sum(v);
      if (t == 0) red[ACT_IMG_THREADS] = rsqrt_f64r(fadd(fdiv(v, (float)a.K), a.eps));
    }
    __syncthreads();
    scale = red[ACT_IMG_THREADS];
    __syncthreads();  // red is reused for the maxima
  }
  // the row's final values (in place) and their largest magnitude
  float mx = 0.0f;
#pragma unroll 1
  for (int i = t, j = 0; i < K4; i += ACT_IMG_THREADS, j++) {
    float4 x = x4[i];
    if (a.gain) {
      float4 g;
      if (greg) {
        g = gr[0];
#pragma unroll
        for (int q = 1; q < GREG; q++)
          if (j == q) g = gr[q];
      } else {
        g = __ldg(reinterpret_cast<const float4*>(a.gain) + i);
      }
      x = make_float4(fmul(fmul(x.x, scale), g.x), fmul(fmul(x.y, scale), g.y),
                      fmul(fmul(x.z, scale), g.z), fmul(fmul(x.w, scale), g.w));
      x4[i] = x;
    }
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((t & 31) == 0) red[t >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const int e = row_exponent(mx);
  if (t == 0) a.row_exp[m] = e;
  // x * 2^-e (exact) rounded to f16, swizzled
  const float sc = pow2f(-e);
  for (int i = t; i < a.K / 8; i += ACT_IMG_THREADS) {
    const float4 x0 = x4[2 * i], x1 = x4[2 * i + 1];
    *reinterpret_cast<uint4*>(base + (size_t)(i >> 3) * a.Nt * 128 + sw128_off(r, i & 7)) =
        make_uint4(h2(x0.x * sc, x0.y * sc), h2(x0.z * sc, x0.w * sc), h2(x1.x * sc, x1.y * sc),
                   h2(x1.z * sc, x1.w * sc));
  }
}

inline int tc_token_tile(int M) {
  const int nt = (M + 15) / 16 * 16;
  return nt < TC_MAX_NT ? nt : TC_MAX_NT;
}

}  // namespace flock
