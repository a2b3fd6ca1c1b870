// Shared device helpers for the flock_b200 kernels (sm_100a).
//
// Numerics contract.  The reference path computes in strict f32 with every
// multiply-add contracted to one FMA and every other operation rounded once
// (kernels/lib.ts:1-21, kernels/ops_ref.ts:1-7).  The kernels here reproduce
// that by writing every rounding explicitly with the _rn intrinsics, which the
// compiler never reassociates or contracts, and the build passes --fmad=false
// so no accidental a*b+c is fused either.  Transcendentals the reference takes
// from f64 libm and rounds to f32 (fr(Math.exp(x)), fr(Math.cos(x)), the
// 1/Math.sqrt of rmsnorm) are evaluated by calling CUDA's double-precision
// functions and rounding once to f32.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#define FLOCK_DEV __device__ __forceinline__

// ------------------------------------------------------------ exact rounding
FLOCK_DEV float fmul(float a, float b) { return __fmul_rn(a, b); }
FLOCK_DEV float fadd(float a, float b) { return __fadd_rn(a, b); }
FLOCK_DEV float fsub(float a, float b) { return __fsub_rn(a, b); }
FLOCK_DEV float ffma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
FLOCK_DEV float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// fr(Math.exp(x)) for an f32 x.
FLOCK_DEV float exp_f64r(float x) { return __double2float_rn(exp((double)x)); }
// fr(1 / Math.sqrt(v)) for an f32 v: IEEE f64 sqrt and divide, one f32 round.
FLOCK_DEV float rsqrt_f64r(float v) { return __double2float_rn(1.0 / sqrt((double)v)); }

// bf16 KV cache elements (FLOCK_KV_BF16): a key or value is rounded to the
// nearest bf16 (ties to even) once, when it is appended, and widened exactly
// (the bf16 bits are the high half of the f32) whenever attention reads it.
FLOCK_DEV uint16_t bf16_bits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
FLOCK_DEV float bf16_round(float x) { return __uint_as_float((uint32_t)bf16_bits(x) << 16); }

// fp8 KV cache elements (FLOCK_KV_FP8): OCP E4M3FN, a key or value rounded to
// the nearest e4m3 (ties to even; magnitudes past 448 saturate to 448) once,
// when it is appended, and widened exactly (e4m3 is a subset of f16) on read.
FLOCK_DEV uint8_t fp8_bits(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
FLOCK_DEV float fp8_widen(uint8_t b) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3)));
}
FLOCK_DEV float fp8_round(float x) { return fp8_widen(fp8_bits(x)); }
// Two e4m3 in the low 16 bits of w -> two f32.
FLOCK_DEV float2 fp8x2_widen(uint32_t w) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xFFFFu), __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
// Sixteen e4m3 (one 128-bit load) -> sixteen f32 at dst (16-byte aligned).
FLOCK_DEV void fp8x16_widen(uint4 w, float* dst) {
  const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 a = fp8x2_widen(v[i]), b = fp8x2_widen(v[i] >> 16);
    reinterpret_cast<float4*>(dst)[i] = make_float4(a.x, a.y, b.x, b.y);
  }
}
// Two bf16 packed in a word (element 0 in the low half) -> two f32.
FLOCK_DEV float2 bf16x2_widen(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
// Eight bf16 (one 128-bit load) -> eight f32 at dst (16-byte aligned).
FLOCK_DEV void bf16x8_widen(uint4 w, float* dst) {
  const float2 a = bf16x2_widen(w.x), b = bf16x2_widen(w.y), c = bf16x2_widen(w.z),
               d = bf16x2_widen(w.w);
  reinterpret_cast<float4*>(dst)[0] = make_float4(a.x, a.y, b.x, b.y);
  reinterpret_cast<float4*>(dst)[1] = make_float4(c.x, c.y, d.x, d.y);
}

// kernels/lib.ts:30 halfToF32: f16 -> f32 exactly, with inf/nan clamped to
// the largest finite f32 (the reference clamps e == 31 regardless of mantissa).
FLOCK_DEV float scale_f16(uint16_t h) {
  if ((h & 0x7C00u) == 0x7C00u) return (h & 0x8000u) ? -FLT_MAX : FLT_MAX;
  return __half2float(__ushort_as_half(h));
}

// Four int8 in a word -> four exact f32.  The bytes are biased to unsigned
// (xor 0x80), placed in the mantissa of 2^23 with a byte permute, and the bias
// 2^23 + 128 subtracted; every step is exact, so the result is (float)(int8).
FLOCK_DEV void dec_i8x4(uint32_t w, float& a, float& b, float& c, float& d) {
  const uint32_t u = w ^ 0x80808080u;
  const float k = 8388736.0f;  // 2^23 + 128
  a = fsub(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u)), k);
  b = fsub(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541u)), k);
  c = fsub(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542u)), k);
  d = fsub(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543u)), k);
}

// Four nibbles already masked to one per byte (0..15) -> exact (q - 8).
FLOCK_DEV void dec_nib4(uint32_t v, float& a, float& b, float& c, float& d) {
  const float k = 8388616.0f;  // 2^23 + 8
  a = fsub(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540u)), k);
  b = fsub(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7541u)), k);
  c = fsub(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7542u)), k);
  d = fsub(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7543u)), k);
}

// kernels/lib.ts:196 dot4: one rounded product, then three FMAs.
FLOCK_DEV float dot4(float q0, float q1, float q2, float q3, float x0, float x1, float x2,
                     float x3) {
  float s = fmul(q0, x0);
  s = ffma(q1, x1, s);
  s = ffma(q2, x2, s);
  s = ffma(q3, x3, s);
  return s;
}

// ------------------------------------------------- packed f32 pairs (sm_100a)
// f32x2 arithmetic rounds each half exactly as the scalar instruction does,
// so two independent chains can share one instruction stream.
FLOCK_DEV uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
FLOCK_DEV float2 unpack2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
FLOCK_DEV uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
FLOCK_DEV uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
FLOCK_DEV uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// ------------------------------------------------------------ memory helpers
FLOCK_DEV uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Fire-and-forget bulk prefetch of [p, p+bytes) into L2 (TMA unit).  p and
// bytes must be 16-byte multiples; callers pass 256-aligned tensor ranges.
FLOCK_DEV void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Programmatic dependent launch.  Everything before pdl_wait() may only read
// memory no earlier kernel in the stream writes (weights); everything that
// reads an activation comes after it.
FLOCK_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FLOCK_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Up to four [ptr, bytes) ranges a kernel prefetches into L2 for the kernel
// after it, split evenly over its CTAs in 32 KiB bulk requests.
struct PrefetchList {
  const uint8_t* ptr[4];
  uint64_t bytes[4];
  int n;
};

FLOCK_DEV void issue_prefetch(const PrefetchList& pf) {
  if (threadIdx.x != 0 || pf.n == 0) return;
  const uint64_t chunk = 32768;
  const uint64_t cta = blockIdx.x + (uint64_t)blockIdx.y * gridDim.x;
  const uint64_t nctas = (uint64_t)gridDim.x * gridDim.y;
  for (int r = 0; r < pf.n; r++) {
    const uint64_t nchunks = (pf.bytes[r] + chunk - 1) / chunk;
    for (uint64_t c = cta; c < nchunks; c += nctas) {
      uint64_t off = c * chunk;
      uint64_t len = pf.bytes[r] - off < chunk ? pf.bytes[r] - off : chunk;
      len &= ~(uint64_t)15;
      if (len) prefetch_l2(pf.ptr[r] + off, (uint32_t)len);
    }
  }
}

// Reference workgroup tree (kernels/lib.ts:312 treeSum) over 32 values held
// one per lane: after the call lane 0 holds buf[0] of the pairwise tree.
FLOCK_DEV float warp_tree_sum(float v) {
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) v = fadd(v, __shfl_down_sync(0xffffffffu, v, s));
  return v;
}
