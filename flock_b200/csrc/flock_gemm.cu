// Host side of the tensor-core prefill GEMM (gemm_tc.cuh): the activation
// image, launches, and the op-level entry points that the M > 1 sweep and
// the parity tests call.
#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "flock_internal.h"
#include "gemm_tc.cuh"

namespace flock {

// The image proper, then one int (the row's scale exponent) per image row.
static size_t act_image_only_bytes(int M, int K) {
  const int nt = tc_token_tile(M);
  const size_t n_mb = (size_t)(M + nt - 1) / nt;
  return n_mb * (size_t)(K / TC_KT) * (size_t)nt * 128;
}

size_t act_image_bytes(int M, int K) {
  const int nt = tc_token_tile(M);
  return act_image_only_bytes(M, K) + (size_t)((M + nt - 1) / nt) * nt * 4;
}

static int act_image_launch(cudaStream_t st, ActImgArgs& a);

int act_image_enqueue(cudaStream_t st, const float* x, int x_stride, const float* gain, float eps,
                      int M, int K, uint8_t* img, const float* atc_part, int atc_nz,
                      int n_heads) {
  if (K % TC_KT || K > 12288 || M < 1) {
    set_error("tensor-core GEMM needs K a multiple of 64 and at most 12288 (K = %d)", K);
    return FLOCK_E_ARG;
  }
  if (atc_part && (atc_nz < 1 || atc_nz > ATC_MAX_SPLITS_IMG || n_heads < 1 || n_heads > 32 ||
                   K % (4 * n_heads))) {
    set_error("attention range merge: %d ranges over %d heads", atc_nz, n_heads);
    return FLOCK_E_ARG;
  }
  ActImgArgs a = {};
  a.x = x;
  a.x_stride = x_stride;
  a.gain = gain;
  a.eps = eps;
  a.M = M;
  a.K = K;
  a.img = img;
  a.part = atc_part;
  a.nz = atc_nz;
  a.n_heads = n_heads;
  return act_image_launch(st, a);
}

int act_image_reduce_enqueue(cudaStream_t st, const float* res, const float* red_part, int red_nz,
                             float* x_out, const float* gain, float eps, int M, int K,
                             uint8_t* img) {
  if (K % TC_KT || K > 12288 || M < 1 || red_nz < 1) return FLOCK_E_ARG;
  ActImgArgs a = {};
  a.x = res;
  a.x_stride = K;
  a.gain = gain;
  a.eps = eps;
  a.M = M;
  a.K = K;
  a.img = img;
  a.red_part = red_part;
  a.red_nz = red_nz;
  a.x_out = x_out;
  return act_image_launch(st, a);
}

int act_image_swiglu_enqueue(cudaStream_t st, const float* gu, int M, int K, uint8_t* img) {
  if (K % TC_KT || K > 12288 || M < 1) return FLOCK_E_ARG;
  ActImgArgs a = {};
  a.x_stride = K;
  a.M = M;
  a.K = K;
  a.img = img;
  a.gu = gu;
  return act_image_launch(st, a);
}

static int act_image_launch(cudaStream_t st, ActImgArgs& a) {
  const int M = a.M, K = a.K;
  a.Nt = tc_token_tile(M);
  a.row_exp = reinterpret_cast<int*>(a.img + act_image_only_bytes(M, K));
  const int rows = (M + a.Nt - 1) / a.Nt * a.Nt;  // image rows, zero past M
  FLOCK_TRY(kernel_setup((const void*)k_act_image, (int)act_image_smem_bytes(12288)));
  FLOCK_CK(launch_ex(st, k_act_image, dim3(rows), dim3(ACT_IMG_THREADS), act_image_smem_bytes(K),
                     true, a));
  return FLOCK_OK;
}

TcSeg tc_seg_of(const flock_tensor* t, float* out, int out_stride) {
  TcSeg s;
  s.qs = t->qs.as<uint8_t>();
  s.sc = t->sc.as<uint16_t>();
  s.sc_stride = t->sc_stride;
  s.rows = (int)t->rows;
  s.out = out;
  s.out_stride = out_stride;
  return s;
}

void tc_finish_tiles(TcArgs& a) {
  int tiles = 0;
  for (int i = 0; i < a.nseg; i++) {
    a.tile0[i] = tiles;
    tiles += (a.seg[i].rows + TC_ROWS - 1) / TC_ROWS;
  }
  a.tile0[a.nseg] = tiles;
}

template <int QT, int EPI>
static int launch_tc(cudaStream_t st, const TcArgs& a, bool defer_reduce) {
  FLOCK_TRY(kernel_setup((const void*)k_gemm_tc<QT, EPI>, TC_SMEM_MAX));
  const size_t smem = gemm_tc_smem_bytes(a.Nt);
  const dim3 grid((unsigned)a.tile0[a.nseg], (unsigned)((a.M + a.Nt - 1) / a.Nt),
                  (unsigned)a.ksplit);
  FLOCK_CK(launch_ex(st, k_gemm_tc<QT, EPI>, grid, dim3(TC_THREADS), smem, true, a));
  if (a.ksplit > 1 && !defer_reduce) {
    const TcSeg& s = a.seg[0];
    const int64_t total = (int64_t)a.M * s.rows;
    FLOCK_CK(launch_ex(st, k_splitk_reduce, dim3((unsigned)((total + 255) / 256)), dim3(256), 0,
                       true, (const float*)a.part, a.ksplit, a.M, s.rows,
                       EPI == EPI_RESIDUAL ? a.res : nullptr, a.res_stride, s.out, s.out_stride));
  }
  return FLOCK_OK;
}

// The TMA tensor map of a qs plane ([rows][row_bytes] uint8, row_bytes = K
// for Q8_0 and K / 2 for Q4_0): box {64 / 32 bytes, 128 rows} with the
// matching 64- / 32-byte swizzle (gemm_tc.cuh tc_read_raw), L2 promotion of
// 256 bytes, zeros past the last row.  Encoded once per (plane, shape) and
// cached: the map is a pure function of those, so a cached entry stays right
// even if a freed plane's address comes back for another tensor.
static int qs_tensor_map(CUtensorMap* out, const uint8_t* qs, int rows, int row_bytes, int qt) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, int, int>, CUtensorMap> cache;
  const auto key = std::make_tuple((const void*)qs, rows, row_bytes, qt);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return FLOCK_OK;
  }
  if (((uintptr_t)qs & 15) || row_bytes % 16 || rows < 1) {
    set_error("tensor-core GEMM: weight plane %p (%d rows of %d bytes) is not TMA-addressable",
              (const void*)qs, rows, row_bytes);
    return FLOCK_E_ARG;
  }
  // the driver's encoder, looked up through the runtime so that loading this
  // library needs no libcuda at link time (the CPU-only build host has none)
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      set_error("cuTensorMapEncodeTiled is not available from the driver");
      return FLOCK_E_CUDA;
    }
    encode = reinterpret_cast<EncodeFn>(fn);
  }
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)(qt == QT_Q8 ? TC_KT : TC_KT / 2), (cuuint32_t)TC_ROWS};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(
      &m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(qs), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE,
      qt == QT_Q8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for a %d x %d weight plane", (int)r, rows,
              row_bytes);
    return FLOCK_E_CUDA;
  }
  cache.emplace(key, m);
  *out = m;
  return FLOCK_OK;
}

// Y = X . W^T for the segments of `a` on the tensor cores; `a.img` must hold
// the activation image of the same M and K.  With `part` (room for
// part_floats) and one segment, a grid too small for the GPU is split along
// K (at least 8 K-tiles per CTA) and reduced by k_splitk_reduce -- or, with
// defer_reduce, left as partials in a.part (a.ksplit of them) for the
// caller's next activation image to sum (act_image_reduce_enqueue).
int gemm_tc_enqueue(cudaStream_t st, int qt, int epi, TcArgs& a, int sm_count,
                    size_t part_floats, bool defer_reduce) {
  if (a.K % TC_KT || a.M < 1 || a.nseg < 1 || a.nseg > 3) return FLOCK_E_ARG;
  for (int i = 0; i < a.nseg; i++)
    FLOCK_TRY(qs_tensor_map(&a.tmap[i], a.seg[i].qs, a.seg[i].rows,
                            qt == QT_Q8 ? a.K : a.K / 2, qt));
  a.img_nt = tc_token_tile(a.M);
  a.row_exp = reinterpret_cast<const int*>(a.img + act_image_only_bytes(a.M, a.K));
  tc_finish_tiles(a);
  // Tokens per CTA: the image tile, or half of it when that still fits the
  // grid in one wave -- twice the CTAs on the small weight matrices, each
  // dequantising its weight tile for half as many tokens.
  a.Nt = a.img_nt;
  if (a.img_nt >= 128 && a.img_nt % 32 == 0 &&
      a.tile0[a.nseg] * ((a.M + a.img_nt / 2 - 1) / (a.img_nt / 2)) <= sm_count)
    a.Nt = a.img_nt / 2;
  a.raw_stages = tc_raw_stages(a.Nt);
  a.ksplit = 1;
  const int ctas = a.tile0[a.nseg] * ((a.M + a.Nt - 1) / a.Nt);
  const int KT = a.K / TC_KT;
  if (a.part && a.nseg == 1 && 2 * ctas <= sm_count) {
    for (int s = 8; s >= 2; s--) {
      if (KT % s || KT / s < 8 || ctas * s > sm_count ||
          (size_t)s * a.M * a.seg[0].rows > part_floats)
        continue;
      a.ksplit = s;
      break;
    }
  }
  if (qt == QT_Q8)
    return epi == EPI_RESIDUAL ? launch_tc<QT_Q8, EPI_RESIDUAL>(st, a, defer_reduce)
                               : launch_tc<QT_Q8, EPI_STORE>(st, a, defer_reduce);
  return epi == EPI_RESIDUAL ? launch_tc<QT_Q4, EPI_RESIDUAL>(st, a, defer_reduce)
                             : launch_tc<QT_Q4, EPI_STORE>(st, a, defer_reduce);
}

}  // namespace flock

using namespace flock;

namespace {

// One op-level GEMM on device buffers: image + tensor-core GEMM; `mid`, when
// given, is recorded between the two kernels.
int gemm_once(flock_dev* d, const flock_tensor* w, const float* x, int M, float* y, int* err,
              uint8_t* img, cudaEvent_t mid = nullptr) {
  const int K = (int)w->cols;
  FLOCK_TRY(act_image_enqueue(d->stream, x, K, nullptr, 0.0f, M, K, img));
  if (mid) FLOCK_CK(cudaEventRecord(mid, d->stream));
  TcArgs a = {};
  a.seg[0] = tc_seg_of(w, y, (int)w->rows);
  a.nseg = 1;
  a.K = K;
  a.M = M;
  a.img = img;
  a.err = err;
  return gemm_tc_enqueue(d->stream, w->dtype == FLOCK_Q8_0 ? QT_Q8 : QT_Q4, EPI_STORE, a,
                         d->sm_count, 0);
}

int check_tc_err(const DBuf& err) {
  int e = 0;
  FLOCK_CK(cudaMemcpy(&e, err.p, 4, cudaMemcpyDeviceToHost));
  if (e) {
    set_error("tensor-core GEMM gave up waiting (code %d)", e);
    return FLOCK_E_CUDA;
  }
  return FLOCK_OK;
}

int gemm_check_args(const flock_tensor* w, int M) {
  if (!w || M < 1 || w->dtype == FLOCK_F32) return FLOCK_E_ARG;
  if (w->cols % TC_KT || w->cols > 12288) {
    set_error("tensor-core GEMM needs cols a multiple of 64 and at most 12288 (cols = %lld)",
              (long long)w->cols);
    return FLOCK_E_ARG;
  }
  return FLOCK_OK;
}

}  // namespace

extern "C" {

int flock_op_gemm(flock_dev* d, const flock_tensor* w, const float* x, int M, float* y) {
  if (!d || !x || !y) return FLOCK_E_ARG;
  FLOCK_TRY(gemm_check_args(w, M));
  FLOCK_CK(cudaSetDevice(d->ordinal));
  DBuf dx, dy, img, err;
  FLOCK_TRY(dx.alloc((size_t)M * w->cols * 4));
  FLOCK_TRY(dy.alloc((size_t)M * w->rows * 4));
  FLOCK_TRY(img.alloc(act_image_bytes(M, (int)w->cols)));
  FLOCK_TRY(err.alloc(16));
  FLOCK_CK(cudaMemset(err.p, 0, 16));
  FLOCK_CK(cudaMemcpy(dx.p, x, dx.bytes, cudaMemcpyHostToDevice));
  FLOCK_TRY(gemm_once(d, w, dx.as<float>(), M, dy.as<float>(), err.as<int>(), img.as<uint8_t>()));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  FLOCK_TRY(check_tc_err(err));
  FLOCK_CK(cudaMemcpy(y, dy.p, dy.bytes, cudaMemcpyDeviceToHost));
  return FLOCK_OK;
}

}  // extern "C"

namespace {

// Bytes written to evict L2 (126 MB on B200) before a cold-timed call.
constexpr size_t kL2FlushBytes = (size_t)256 << 20;

int gemm_timed(flock_dev* d, const flock_tensor* w, int M, int iters, bool cold,
               float* ms_per_call, float* ms_image) {
  if (!d || iters < 1 || !ms_per_call || !ms_image) return FLOCK_E_ARG;
  FLOCK_TRY(gemm_check_args(w, M));
  FLOCK_CK(cudaSetDevice(d->ordinal));
  std::vector<float> hx((size_t)M * w->cols);
  uint32_t s = 777u;
  for (auto& v : hx) {  // xorshift32 in [-1, 1)
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    v = (float)((double)s / 2147483648.0 - 1.0);
  }
  DBuf dx, dy, img, err;
  FLOCK_TRY(dx.alloc(hx.size() * 4));
  FLOCK_TRY(dy.alloc((size_t)M * w->rows * 4));
  FLOCK_TRY(img.alloc(act_image_bytes(M, (int)w->cols)));
  FLOCK_TRY(err.alloc(16));
  FLOCK_CK(cudaMemset(err.p, 0, 16));
  FLOCK_CK(cudaMemcpy(dx.p, hx.data(), dx.bytes, cudaMemcpyHostToDevice));
  DBuf flush;
  if (cold) FLOCK_TRY(flush.alloc(kL2FlushBytes));
  FLOCK_TRY(gemm_once(d, w, dx.as<float>(), M, dy.as<float>(), err.as<int>(), img.as<uint8_t>()));
  // per call: [start] image [mid] GEMM [end], each pair timed on the device
  std::vector<cudaEvent_t> ev(3 * (size_t)iters, nullptr);
  int rc = FLOCK_OK;
  auto ck = [&](cudaError_t e) {
    if (e != cudaSuccess && !rc) {
      set_error("CUDA error %s in the timed GEMM loop", cudaGetErrorString(e));
      rc = FLOCK_E_CUDA;
    }
  };
  for (auto& e : ev) ck(cudaEventCreate(&e));
  for (int i = 0; i < iters && !rc; i++) {
    if (cold) ck(cudaMemsetAsync(flush.p, i & 0xff, flush.bytes, d->stream));
    ck(cudaEventRecord(ev[3 * i], d->stream));
    if (!rc)
      rc = gemm_once(d, w, dx.as<float>(), M, dy.as<float>(), err.as<int>(), img.as<uint8_t>(),
                     ev[3 * i + 1]);
    ck(cudaEventRecord(ev[3 * i + 2], d->stream));
  }
  float gemm = 0, image = 0;
  if (!rc) {
    ck(cudaStreamSynchronize(d->stream));
    for (int i = 0; i < iters && !rc; i++) {
      float a = 0, b = 0;
      ck(cudaEventElapsedTime(&a, ev[3 * i], ev[3 * i + 1]));
      ck(cudaEventElapsedTime(&b, ev[3 * i + 1], ev[3 * i + 2]));
      image += a;
      gemm += b;
    }
  }
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  FLOCK_TRY(rc);
  *ms_per_call = gemm / iters;
  *ms_image = image / iters;
  return check_tc_err(err);
}

}  // namespace

extern "C" {

int flock_op_gemm_timed(flock_dev* d, const flock_tensor* w, int M, int iters, float* ms_per_call,
                        float* ms_image) {
  return gemm_timed(d, w, M, iters, false, ms_per_call, ms_image);
}

int flock_op_gemm_timed_cold(flock_dev* d, const flock_tensor* w, int M, int iters,
                             float* ms_per_call, float* ms_image) {
  return gemm_timed(d, w, M, iters, true, ms_per_call, ms_image);
}

}  // extern "C"
