// libflock_cuda.so: devices, tensors, launch planning and the op-level,
// Layer and range entry points of include/flock_cuda.h.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstring>
#include <string>
#include <mutex>
#include <map>
#include <vector>

// decode o_proj / down: store + separate residual add from this hidden size up
#ifndef FLOCK_SPLIT_RESIDUAL_MIN_HIDDEN
#define FLOCK_SPLIT_RESIDUAL_MIN_HIDDEN 4096
#endif

#include "attn_fast.cuh"
#include "attn_tc.cuh"
#include "gemm_tc.cuh"
#include "flock_internal.h"
#include "gemv.cuh"
#include "gemv_fast.cuh"
#include "ops.cuh"

namespace flock {

static thread_local std::string g_err;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
}

int DBuf::alloc(size_t n) {
  release();
  if (n == 0) n = 16;
  cudaError_t e = cudaMalloc(&p, n);
  if (e != cudaSuccess) {
    p = nullptr;
    set_error("cudaMalloc(%zu) failed: %s", n, cudaGetErrorString(e));
    return FLOCK_E_NOMEM;
  }
  bytes = n;
  return FLOCK_OK;
}

void DBuf::release() {
  if (p) cudaFree(p);
  p = nullptr;
  bytes = 0;
}

const char* const kTensorNames[W_COUNT] = {
    "attn_q.weight",   "attn_k.weight",    "attn_v.weight",      "attn_output.weight",
    "ffn_gate.weight", "ffn_up.weight",    "ffn_down.weight",    "attn_norm.weight",
    "attn_q_norm.weight", "attn_k_norm.weight", "ffn_norm.weight"};

// ------------------------------------------------------------- launching

int kernel_setup(const void* func, int max_dyn_smem, int carveout) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> opted;  // largest opt-in so far
  int dev = 0;
  FLOCK_CK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  auto it = opted.find({func, dev});
  if (it != opted.end() && it->second >= max_dyn_smem) return FLOCK_OK;
  if (max_dyn_smem > 0)
    FLOCK_CK(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, max_dyn_smem));
  if (carveout >= 0)
    FLOCK_CK(cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, carveout));
  opted[{func, dev}] = max_dyn_smem;
  return FLOCK_OK;
}


// SwiGLU (gate/up) rows of one block per lane run three CTAs per SM: its
// 2 x ffn rows at two per warp step are more row groups than two CTAs per
// SM have warps, and a warp's second group loads its weights only after the
// dependency wait; at three (x pairs read per step from shared memory, so
// the registers fit) every warp has one group (3072 rows: 665 against 678
// us per 0.6B-shape token)
constexpr int GEMV_SWIGLU_CTAS_PER_SM = 3;
static bool gemv_swiglu3(int EPI, int K, int LA) { return EPI == EPI_SWIGLU && K <= 1024 && LA == 1; }

template <int QT, int R, int EPI, int MX, int LA = 1>
static cudaError_t gemv_go(flock_dev* d, const GemvArgs& a, int ctas, bool pdl) {
  if (gemv_swiglu3(EPI, a.K, LA)) {
    auto k3 = k_gemv<QT, R, EPI, MX, LA, GEMV_SWIGLU_CTAS_PER_SM, 2>;
    const size_t smem3 = gemv_smem_bytes(a.K, a.norm_gain != nullptr);
    if (kernel_setup((const void*)k3, 200 * 1024)) return cudaErrorInvalidValue;
    return launch_ex(d->stream, k3, dim3(ctas, a.n_tokens), dim3(GEMV_THREADS), smem3, pdl, a);
  }
  // blocks fold on f32x2 pairs (x staged in the packed-pair layout): held in
  // registers for one-block rows, read per step otherwise; two rows with two
  // steps in flight keep the scalar fold (the pairs would spill)
  auto k = a.K <= 1024 ? (LA == 1 ? k_gemv<QT, R, EPI, MX, LA, 2, 1>
                                  : k_gemv<QT, R, EPI, MX, LA, 2, 0>)
                       : ((R == 1 || LA == 1) ? k_gemv<QT, R, EPI, MX, LA, 2, 2>
                                              : k_gemv<QT, R, EPI, MX, LA, 2, 0>);
  const size_t smem = gemv_smem_bytes(a.K, a.norm_gain != nullptr);
  if (kernel_setup((const void*)k, 200 * 1024)) return cudaErrorInvalidValue;
  return launch_ex(d->stream, k, dim3(ctas, a.n_tokens), dim3(GEMV_THREADS), smem, pdl, a);
}

int gemv_grid(flock_dev* d, int total_groups) {
  int ctas = (total_groups + GEMV_WARPS - 1) / GEMV_WARPS;
  const int cap = 2 * d->sm_count;
  return ctas < 1 ? 1 : (ctas > cap ? cap : ctas);
}

int launch_gemv(flock_dev* d, int QT, int EPI, const GemvArgs& a, bool pdl) {
  if (a.K % 32 != 0 || a.K > 24576 || (a.norm_gain && a.K > 12288)) {
    set_error("matvec cols %d must be a multiple of 32 and <= 24576 (12288 with a fused norm)",
              a.K);
    return FLOCK_E_ARG;
  }
  const int M = (a.K / 32 + 31) / 32;
  int rows = 0;
  for (int s = 0; s < a.nseg; s++) rows += a.seg[s].rows;
  // large matrices with long rows (the 8B shape): two rows per warp step and
  // one step of lookahead on the f32x2 fold measured fastest (4096 x 12288:
  // 16.4 us against 20.7 for one row with two steps in flight)
  const bool big = a.K > 1024 && rows >= 4096;
  // steps of weights in flight: two for long rows, else one
  const int MX = (M >= 2 && !big) ? 2 : 1;
  // rows per warp step: 2 where that keeps one wave of <= 2 CTAs per SM busy
  // with about one row group per warp, 1 for the small matrices
  int R = 1;
  if (EPI == EPI_SWIGLU || EPI == EPI_ARGMAX || big) R = 2;
  else if (EPI == EPI_STORE && rows > 2 * GEMV_WARPS * d->sm_count) R = 2;
  int groups;
  if (EPI == EPI_SWIGLU) groups = a.seg[0].rows;
  else {
    groups = 0;
    for (int s = 0; s < a.nseg; s++) groups += (a.seg[s].rows + R - 1) / R;
  }
  // rows of 2-3 column blocks per lane in small matrices (the 0.6B o_proj,
  // down): one row per warp pair (k_gemv_pair, the same arithmetic)
  if (QT == QT_Q8 && (EPI == EPI_STORE || EPI == EPI_RESIDUAL) && a.nseg == 1 && !big &&
      (M == 2 || M == 3) && a.K <= 12288) {
    const int pctas = (rows + GEMV_PAIRS - 1) / GEMV_PAIRS;
    if (pctas <= 2 * d->sm_count) {
      auto k = EPI == EPI_STORE ? k_gemv_pair<QT_Q8, EPI_STORE> : k_gemv_pair<QT_Q8, EPI_RESIDUAL>;
      const size_t smem = gemv_pair_smem_bytes(a.K, a.norm_gain != nullptr);
      if (kernel_setup((const void*)k, 200 * 1024)) return FLOCK_E_CUDA;
      cudaError_t pe = launch_ex(d->stream, k, dim3(pctas, a.n_tokens), dim3(GEMV_THREADS), smem,
                                 pdl, a);
      if (pe != cudaSuccess) {
        set_error("matvec launch failed: %s", cudaGetErrorString(pe));
        return FLOCK_E_CUDA;
      }
      return FLOCK_OK;
    }
  }
  int ctas = gemv_grid(d, groups);
  if (gemv_swiglu3(EPI, a.K, MX == 1 ? 1 : 2)) {
    ctas = (groups + GEMV_WARPS - 1) / GEMV_WARPS;
    if (ctas > GEMV_SWIGLU_CTAS_PER_SM * d->sm_count) ctas = GEMV_SWIGLU_CTAS_PER_SM * d->sm_count;
  }
  cudaError_t e = cudaErrorInvalidValue;
// long rows (two or more column blocks per lane) keep one x block in
// registers and two steps of weights in flight; short rows keep the x
// blocks and one step
#define GO(qt, r, epi, mx) \
  e = (mx) == 1 ? gemv_go<qt, r, epi, 1, 1>(d, a, ctas, pdl) : gemv_go<qt, r, epi, 1, 2>(d, a, ctas, pdl)
  if (QT == QT_Q8) {
    switch (EPI) {
      case EPI_STORE:
        if (R == 2) { if (MX == 1) GO(QT_Q8, 2, EPI_STORE, 1); else GO(QT_Q8, 2, EPI_STORE, 2); }
        else { if (MX == 1) GO(QT_Q8, 1, EPI_STORE, 1); else GO(QT_Q8, 1, EPI_STORE, 2); }
        break;
      case EPI_RESIDUAL:
        if (R == 2) { if (MX == 1) GO(QT_Q8, 2, EPI_RESIDUAL, 1); else GO(QT_Q8, 2, EPI_RESIDUAL, 2); }
        else { if (MX == 1) GO(QT_Q8, 1, EPI_RESIDUAL, 1); else GO(QT_Q8, 1, EPI_RESIDUAL, 2); }
        break;
      case EPI_SWIGLU:
        if (MX == 1) GO(QT_Q8, 2, EPI_SWIGLU, 1); else GO(QT_Q8, 2, EPI_SWIGLU, 2);
        break;
      case EPI_ARGMAX:
        if (MX == 1) GO(QT_Q8, 2, EPI_ARGMAX, 1); else GO(QT_Q8, 2, EPI_ARGMAX, 2);
        break;
    }
  } else {
    if (EPI != EPI_STORE) {
      set_error("Q4_0 matvec supports the plain store epilogue only");
      return FLOCK_E_UNSUPPORTED;
    }
    if (R == 2) { if (MX == 1) GO(QT_Q4, 2, EPI_STORE, 1); else GO(QT_Q4, 2, EPI_STORE, 2); }
    else { if (MX == 1) GO(QT_Q4, 1, EPI_STORE, 1); else GO(QT_Q4, 1, EPI_STORE, 2); }
  }
#undef GO
  if (e != cudaSuccess) {
    set_error("matvec launch failed: %s", cudaGetErrorString(e));
    return FLOCK_E_CUDA;
  }
  return FLOCK_OK;
}

template <int QT, int EPI>
static cudaError_t gemv_fast_go(flock_dev* d, const GemvArgs& a, int ctas, bool pdl) {
  auto k = k_gemv_fast<QT, EPI>;
  const size_t smem = gemv_fast_smem_bytes(a.K, a.norm_gain != nullptr);
  if (kernel_setup((const void*)k, 200 * 1024)) return cudaErrorInvalidValue;
  return launch_ex(d->stream, k, dim3(ctas, a.n_tokens), dim3(GEMV_THREADS), smem, pdl, a);
}

int launch_gemv_fast(flock_dev* d, int QT, int EPI, const GemvArgs& a, bool pdl) {
  if (a.K % 32 != 0 || a.K > 12288 || a.n_tokens < 1) {
    set_error("fast matvec cols %d must be a multiple of 32 and <= 12288", a.K);
    return FLOCK_E_ARG;
  }
  int groups = 0;
  for (int s = 0; s < a.nseg; s++) groups += (a.seg[s].rows + GF_ROWS - 1) / GF_ROWS;
  const int ctas = gemv_grid(d, groups);
  cudaError_t e = cudaErrorInvalidValue;
  if (QT == QT_Q8 && EPI == EPI_STORE) e = gemv_fast_go<QT_Q8, EPI_STORE>(d, a, ctas, pdl);
  else if (QT == QT_Q8 && EPI == EPI_RESIDUAL) e = gemv_fast_go<QT_Q8, EPI_RESIDUAL>(d, a, ctas, pdl);
  else if (QT == QT_Q8 && EPI == EPI_ARGMAX) e = gemv_fast_go<QT_Q8, EPI_ARGMAX>(d, a, ctas, pdl);
  else if (QT == QT_Q4 && EPI == EPI_STORE) e = gemv_fast_go<QT_Q4, EPI_STORE>(d, a, ctas, pdl);
  else {
    set_error("the fast matvec has the store, residual and argmax epilogues (Q4_0: store)");
    return FLOCK_E_UNSUPPORTED;
  }
  if (e != cudaSuccess) {
    set_error("fast matvec launch failed: %s", cudaGetErrorString(e));
    return FLOCK_E_CUDA;
  }
  return FLOCK_OK;
}

static GemvSeg seg_of(const flock_tensor* t, float* out, int out_stride) {
  GemvSeg s;
  s.qs = t->qs.as<uint8_t>();
  s.sc = t->sc.as<uint16_t>();
  s.out = out;
  s.rows = (int)t->rows;
  s.sc_stride = t->sc_stride;
  s.out_stride = out_stride;
  return s;
}

// L2 prefetch hints for the next kernel's weights.  A tensor larger than
// kPrefetchMax is left to stream on demand: prefetching it would compete with
// the running kernel's own HBM stream and could be evicted before its use
// (the 8B shape's 50 MB gate / up / down planes next to a 126 MB L2).
constexpr uint64_t kPrefetchMax = 24ull << 20;
static void pf_add(PrefetchList& pf, const flock_tensor* t) {
  if (!t || t->qs.bytes > kPrefetchMax) return;
  if (pf.n + 2 > 4) return;
  pf.ptr[pf.n] = t->qs.as<uint8_t>();
  pf.bytes[pf.n] = t->qs.bytes & ~(uint64_t)15;
  pf.n++;
  pf.ptr[pf.n] = t->sc.as<uint8_t>();
  pf.bytes[pf.n] = t->sc.bytes & ~(uint64_t)15;
  pf.n++;
}

// ------------------------------------------------------------ device refs

flock_dev* dev_retain(flock_dev* d) {
  if (d) d->refs.fetch_add(1, std::memory_order_relaxed);
  return d;
}

void dev_release(flock_dev* d) {
  if (!d || d->refs.fetch_sub(1, std::memory_order_acq_rel) != 1) return;
  cudaSetDevice(d->ordinal);
  cudaStreamSynchronize(d->stream);
  cudaEventDestroy(d->t0);
  cudaEventDestroy(d->t1);
  cudaStreamDestroy(d->stream);
  delete d;
}

// ------------------------------------------------------------- workspace

int Workspace::alloc(const flock_layer_config& c, int sm_count, int tp_ranks) {
  P = c.max_prefill < 1 ? 1 : c.max_prefill;
  attn_splits = attn_max_splits(sm_count, c.n_kv_heads, c.max_keys);
  H = c.hidden;
  nH = c.n_heads;
  nKV = c.n_kv_heads;
  hd = c.head_dim;
  F = c.ffn;
  const size_t f = sizeof(float);
  FLOCK_TRY(h.alloc((size_t)P * H * f));
  FLOCK_TRY(q.alloc((size_t)P * nH * hd * f));
  FLOCK_TRY(k.alloc((size_t)P * nKV * hd * f));
  FLOCK_TRY(v.alloc((size_t)P * nKV * hd * f));
  FLOCK_TRY(qn.alloc((size_t)P * nH * hd * f));
  FLOCK_TRY(attn.alloc((size_t)P * nH * hd * f));
  FLOCK_TRY(act.alloc((size_t)P * F * f));
  FLOCK_TRY(attn_part.alloc((size_t)nH * attn_splits * (hd + 2) * f));  // stride: attn_splits
  FLOCK_TRY(attn_count.alloc((size_t)nKV * 4));
  FLOCK_CK(cudaMemset(attn_count.p, 0, attn_count.bytes));
  if (hd == 128) {
    // the RoPE (cos, sin) of every position the cache holds, the values
    // norm_rope_warp evaluates in f64 (layer.ts:180 inv_freq, as layer_init
    // computes it)
    std::vector<float> inv(hd / 2);
    for (int j = 0; j < hd / 2; j++)
      inv[j] = (float)(1.0 / std::pow(c.rope_base, (double)(2 * j) / (double)hd));
    DBuf dinv;
    FLOCK_TRY(dinv.alloc(inv.size() * sizeof(float)));
    FLOCK_CK(cudaMemcpy(dinv.p, inv.data(), inv.size() * sizeof(float), cudaMemcpyHostToDevice));
    rope_rows = c.max_keys < 1 ? 1 : c.max_keys;
    FLOCK_TRY(rope.alloc((size_t)rope_rows * 64 * sizeof(float2)));
    k_rope_table<<<(rope_rows * 64 + 255) / 256, 256>>>(dinv.as<float>(), rope_rows,
                                                        rope.as<float2>());
    FLOCK_CK(cudaGetLastError());
    FLOCK_CK(cudaDeviceSynchronize());
  }
  if (c.prefill == FLOCK_PREFILL_TENSOR) {
    size_t ib = act_image_bytes(P, H);
    const size_t iq = act_image_bytes(P, nH * hd), iff = act_image_bytes(P, F);
    ib = ib > iq ? ib : iq;
    ib = ib > iff ? ib : iff;
    FLOCK_TRY(img.alloc(ib));
    FLOCK_TRY(gu.alloc((size_t)P * 2 * F * f));
    FLOCK_TRY(tc_err.alloc(16));
    FLOCK_CK(cudaMemset(tc_err.p, 0, 16));
    FLOCK_TRY(part.alloc((size_t)8 * P * H * f));
    FLOCK_TRY(kv_img.alloc(kv_image_bytes(c.max_keys, nKV)));
    FLOCK_CK(cudaMemset(kv_img.p, 0, kv_img.bytes));  // entries past a step's keys stay finite
    FLOCK_TRY(atc_part.alloc((size_t)ATC_MAX_SPLITS * P * nH * (hd + 2) * f));
    q_tiles = (P + ATC_Q - 1) / ATC_Q;
    FLOCK_TRY(q_img.alloc((size_t)nH * q_tiles * ATC_OPND));
    FLOCK_CK(cudaMemset(q_img.p, 0, q_img.bytes));  // rows past a step's queries stay finite
  }
  if (tp_ranks >= 1 || H >= FLOCK_SPLIT_RESIDUAL_MIN_HIDDEN)  // also the split residual
    FLOCK_TRY(tp_part.alloc((size_t)P * H * f));
  if (tp_ranks >= 1) FLOCK_TRY(tp_all.alloc((size_t)tp_ranks * P * H * f));
  return FLOCK_OK;
}

// --------------------------------------------------------------- layer

static int check_cfg(const flock_layer_config& c) {
  if (c.head_dim != 128) {
    set_error("head_dim %d: the kernels are built for head_dim 128", c.head_dim);
    return FLOCK_E_UNSUPPORTED;
  }
  if (c.hidden % 32 || c.ffn % 32 || c.hidden < 32 || c.ffn < 32) {
    set_error("hidden %d and ffn %d must be multiples of 32", c.hidden, c.ffn);
    return FLOCK_E_ARG;
  }
  if (c.n_kv_heads < 1 || c.n_heads % c.n_kv_heads) {
    set_error("n_heads %d must be a multiple of n_kv_heads %d", c.n_heads, c.n_kv_heads);
    return FLOCK_E_ARG;
  }
  if (c.n_heads / c.n_kv_heads > 4) {
    set_error("GQA group size %d > 4 is not supported", c.n_heads / c.n_kv_heads);
    return FLOCK_E_UNSUPPORTED;
  }
  if (c.max_keys < 1 || c.max_prefill < 1) {
    set_error("max_keys and max_prefill must be >= 1");
    return FLOCK_E_ARG;
  }
  if (c.prefill != FLOCK_PREFILL_EXACT && c.prefill != FLOCK_PREFILL_TENSOR) {
    set_error("prefill mode %d is neither FLOCK_PREFILL_EXACT nor FLOCK_PREFILL_TENSOR", c.prefill);
    return FLOCK_E_ARG;
  }
  if (c.prefill == FLOCK_PREFILL_TENSOR &&
      (c.hidden % 64 || c.ffn % 64 || c.hidden > 12288 || c.ffn > 12288)) {
    set_error("tensor-core prefill needs hidden %d and ffn %d multiples of 64, at most 12288", c.hidden,
              c.ffn);
    return FLOCK_E_UNSUPPORTED;
  }
  if (c.kv_dtype != FLOCK_KV_F32 && c.kv_dtype != FLOCK_KV_BF16 && c.kv_dtype != FLOCK_KV_FP8) {
    set_error("kv_dtype %d is not FLOCK_KV_F32, FLOCK_KV_BF16 or FLOCK_KV_FP8", c.kv_dtype);
    return FLOCK_E_ARG;
  }
  if (c.matvec != FLOCK_MATVEC_EXACT && c.matvec != FLOCK_MATVEC_FAST) {
    set_error("matvec %d is neither FLOCK_MATVEC_EXACT nor FLOCK_MATVEC_FAST", c.matvec);
    return FLOCK_E_ARG;
  }
  if (c.kv_dtype != FLOCK_KV_F32 &&
      (c.attention != FLOCK_ATTN_FAST || c.prefill != FLOCK_PREFILL_TENSOR)) {
    set_error("a %s KV cache needs FLOCK_ATTN_FAST and FLOCK_PREFILL_TENSOR (the exact "
              "kernels read f32)", c.kv_dtype == FLOCK_KV_BF16 ? "bf16" : "fp8");
    return FLOCK_E_UNSUPPORTED;
  }
  if (c.attention == FLOCK_ATTN_EXACT && c.max_keys > 48 * 1024) {
    set_error("exact decode attention holds every score on chip: max_keys %d > 49152; use "
              "FLOCK_ATTN_FAST", c.max_keys);
    return FLOCK_E_UNSUPPORTED;
  }
  return FLOCK_OK;
}

int layer_init(flock_layer* L, flock_dev* dev, const flock_layer_config& cfg, Workspace* ws,
               int* shared_ctl) {
  FLOCK_TRY(check_cfg(cfg));
  L->dev = dev_retain(dev);
  L->cfg = cfg;
  const size_t kv = (size_t)cfg.max_keys * cfg.n_kv_heads * cfg.head_dim * kv_elem_bytes(cfg);
  FLOCK_TRY(L->kcache.alloc(kv));
  FLOCK_TRY(L->vcache.alloc(kv));
  std::vector<float> inv(cfg.head_dim / 2);
  // layer.ts:180 invFreqOf: fr(1 / base^(2j/headDim)), on the host.
  for (int j = 0; j < cfg.head_dim / 2; j++)
    inv[j] = (float)(1.0 / std::pow(cfg.rope_base, (double)(2 * j) / (double)cfg.head_dim));
  FLOCK_TRY(L->inv_freq.alloc(inv.size() * sizeof(float)));
  FLOCK_CK(cudaMemcpy(L->inv_freq.p, inv.data(), inv.size() * sizeof(float),
                      cudaMemcpyHostToDevice));
  if (shared_ctl) {
    L->ctl = shared_ctl;
  } else {
    FLOCK_TRY(L->ctl_own.alloc(2 * sizeof(int)));
    FLOCK_CK(cudaMemset(L->ctl_own.p, 0, 2 * sizeof(int)));
    L->ctl = L->ctl_own.as<int>();
  }
  if (ws) {
    L->ws = ws;
  } else {
    FLOCK_TRY(L->ws_own.alloc(cfg, dev->sm_count));
    L->ws = &L->ws_own;
    L->owns_ws = true;
  }
  return FLOCK_OK;
}

// q/k norm + RoPE + KV append, then attention over n >= 1 queries: in
// attnRef / attnPrefillRef order, or (tensor_cores, n > 1) on tcgen05.
static int enqueue_qk_attn(flock_layer* L, int n, bool pdl, bool tensor_cores) {
  flock_dev* d = L->dev;
  Workspace* ws = L->ws;
  const flock_layer_config& c = L->cfg;
  QkArgs qa = {};
  qa.q = ws->q.as<float>();
  qa.k = ws->k.as<float>();
  qa.v = ws->v.as<float>();
  qa.q_norm = L->w[W_Q_NORM]->data.as<float>();
  qa.k_norm = L->w[W_K_NORM]->data.as<float>();
  qa.inv_freq = L->inv_freq.as<float>();
  qa.qn = ws->qn.as<float>();
  qa.kcache = L->kcache.p;
  qa.vcache = L->vcache.p;
  qa.ctl = L->ctl;
  qa.n_tokens = n;
  qa.n_heads = c.n_heads;
  qa.n_kv_heads = c.n_kv_heads;
  qa.head_dim = c.head_dim;
  qa.eps = c.eps;
  qa.neox = c.rope_pairing == FLOCK_ROPE_NEOX;
  pf_add(qa.pf, L->w[W_GATE]);
  const int img_tiles = (c.max_keys + ATC_K - 1) / ATC_K;
  if (n > 1 && tensor_cores) {
    qa.kv_img = ws->kv_img.as<uint8_t>();
    qa.img_tiles = img_tiles;
    qa.q_img = ws->q_img.as<uint8_t>();
    qa.q_tiles = ws->q_tiles;
  }
  qa.rope_cs = ws->rope.as<float2>();
  qa.rope_rows = ws->rope_rows;
  const int kv = c.kv_dtype;
  if (kv != FLOCK_KV_F32 && !(n > 1 && tensor_cores)) {
    set_error("a %s KV cache runs decode on FLOCK_ATTN_FAST and prefill on the tensor cores",
              kv == FLOCK_KV_BF16 ? "bf16" : "fp8");
    return FLOCK_E_UNSUPPORTED;
  }
  FLOCK_CK(launch_ex(d->stream,
                     kv == FLOCK_KV_FP8 ? k_qk_norm_rope_append<FLOCK_KV_FP8>
                     : kv == FLOCK_KV_BF16 ? k_qk_norm_rope_append<FLOCK_KV_BF16>
                                           : k_qk_norm_rope_append<FLOCK_KV_F32>,
                     dim3((n * (c.n_heads + c.n_kv_heads) + 7) / 8), dim3(256), 0, pdl, qa));
  AttnArgs aa = {};
  aa.q = ws->qn.as<float>();
  aa.kcache = L->kcache.as<float>();
  aa.vcache = L->vcache.as<float>();
  aa.out = ws->attn.as<float>();
  aa.ctl = L->ctl;
  aa.n_tokens = n;
  aa.n_heads = c.n_heads;
  aa.n_kv_heads = c.n_kv_heads;
  aa.head_dim = c.head_dim;
  pf_add(aa.pf, L->w[W_UP]);
  if (n > 1 && tensor_cores) {
    // the f16 image of the keys cached before this step (pos0 is read on
    // the device; the new keys went into the image with the append); a
    // step from an empty cache has none
    if (L->n_keys > 0) {
      auto* kvi = kv == FLOCK_KV_FP8 ? k_kv_image<FLOCK_KV_FP8>
                  : kv == FLOCK_KV_BF16 ? k_kv_image<FLOCK_KV_BF16> : k_kv_image<FLOCK_KV_F32>;
      FLOCK_TRY(kernel_setup((const void*)kvi, (int)kv_image_smem_bytes()));
      const int old_tiles = (L->n_keys + ATC_K - 1) / ATC_K;
      FLOCK_CK(launch_ex(d->stream, kvi,
                         dim3(old_tiles < img_tiles ? old_tiles : img_tiles, c.n_kv_heads),
                         dim3(ATC_THREADS), kv_image_smem_bytes(), true,
                         (const void*)L->kcache.p, (const void*)L->vcache.p, c.n_kv_heads,
                         (const int*)L->ctl, n, img_tiles, ws->kv_img.as<uint8_t>()));
    }
    AttnTcArgs ta = {};
    ta.q = ws->qn.as<float>();
    ta.kv_img = ws->kv_img.as<uint8_t>();
    ta.img_tiles = img_tiles;
    ta.out = ws->attn.as<float>();
    ta.ctl = L->ctl;
    ta.n_tokens = n;
    ta.n_heads = c.n_heads;
    ta.n_kv_heads = c.n_kv_heads;
    ta.err = ws->tc_err.as<int>();
    ta.part = ws->atc_part.as<float>();
    ta.q_img = ws->q_img.as<uint8_t>();
    ta.q_tiles = ws->q_tiles;
    // key ranges: sized from the host's count of cached keys (the kernel
    // reads pos0 on the device; a range past its query tile's keys is empty)
    const int nz = attn_tc_splits(L->n_keys, n);
    FLOCK_TRY(kernel_setup((const void*)k_attn_prefill_tc, (int)attn_tc_smem_bytes()));
    FLOCK_CK(launch_ex(d->stream, k_attn_prefill_tc, dim3((n + ATC_Q - 1) / ATC_Q, c.n_heads, nz),
                       dim3(ATC_THREADS), attn_tc_smem_bytes(), true, ta));
    // with several key ranges the o_proj activation image merges them
    // (act_image_enqueue); ws->attn is then not written
    ws->atc_nz = nz;
  } else if (n == 1) {
    const size_t smem = (size_t)c.max_keys * sizeof(float);
    FLOCK_TRY(kernel_setup((const void*)k_attn_decode_exact, 200 * 1024));
    FLOCK_CK(launch_ex(d->stream, k_attn_decode_exact, dim3(c.n_heads), dim3(256), smem, pdl,
                       aa));
  } else {
    FLOCK_CK(launch_ex(d->stream, k_attn_prefill_exact, dim3(c.n_heads, n), dim3(128), 0, pdl,
                       aa));
  }
  return FLOCK_OK;
}

// Tensor parallel: h[i] += (p_0[i] + p_1[i] + ... + p_{N-1}[i]), the ranks'
// partials summed serially in rank order (shard_ref.ts / shard_reduce.wgsl:47
// order), then added to the residual as the unsharded epilogue adds o.
static __global__ void k_tp_reduce_residual(float* h, const float* parts, int n_ranks,
                                            int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = parts[i];
  for (int r = 1; r < n_ranks; r++) acc = fadd(acc, parts[(int64_t)r * n + i]);
  h[i] = fadd(h[i], acc);
}

static int tp_sum_into_h(flock_layer* L, int n) {
  Workspace* ws = L->ws;
  if (!ws->tp_part.p || !ws->tp_all.p || n > ws->P) {
    set_error("tensor-parallel layer without its exchange buffers");
    return FLOCK_E_STATE;
  }
  const int64_t count = (int64_t)n * L->cfg.hidden;
  if (L->xchg && n == 1)  // decode: the fused peer-memory exchange, same sum
    return peer_xchg_run(L->xchg, L->dev->stream, ws->h.as<float>(), ws->tp_part.as<float>(),
                         count);
  FLOCK_TRY(comm_allgather_dev(L->tp, ws->tp_part.p, ws->tp_all.p, (size_t)count * 4));
  k_tp_reduce_residual<<<(unsigned)((count + 255) / 256), 256, 0, L->dev->stream>>>(
      ws->h.as<float>(), ws->tp_all.as<float>(), L->tp_n, count);
  FLOCK_CK(cudaGetLastError());
  return FLOCK_OK;
}

// Large decode shapes (hidden >= 4096): o_proj / down store their result and
// a separate kernel adds it to h -- the residual epilogue's fadd(h, y) --
// which measured faster than the in-epilogue residual at these sizes.
static bool split_residual(const flock_layer* L, int n) {
  return !L->tp && n == 1 && L->cfg.hidden >= FLOCK_SPLIT_RESIDUAL_MIN_HIDDEN && L->ws->tp_part.p;
}
static int add_split_residual(flock_layer* L, int n) {
  const int64_t count = (int64_t)n * L->cfg.hidden;
  k_tp_reduce_residual<<<(unsigned)((count + 255) / 256), 256, 0, L->dev->stream>>>(
      L->ws->h.as<float>(), L->ws->tp_part.as<float>(), 1, count);
  FLOCK_CK(cudaGetLastError());
  return FLOCK_OK;
}

// One prefill step of n > 1 tokens with the four weight matmuls on the
// tcgen05 tensor cores (FLOCK_PREFILL_TENSOR); norms, RoPE, attention and the
// residual adds keep their f32 arithmetic.
static int layer_enqueue_tc(flock_layer* L, int n, bool advance) {
  flock_dev* d = L->dev;
  Workspace* ws = L->ws;
  const flock_layer_config& c = L->cfg;
  cudaStream_t st = d->stream;
  const int qw = c.n_heads * c.head_dim, kvw = c.n_kv_heads * c.head_dim, H = c.hidden,
            F = c.ffn;
  uint8_t* img = ws->img.as<uint8_t>();
  int* err = ws->tc_err.as<int>();
  int o_split = 1;  // K-splits of the o_proj GEMM whose partials the ffn image sums
  if (advance) {
    k_ctl_advance<<<1, 1, 0, st>>>(L->ctl, n);
    FLOCK_CK(cudaGetLastError());
  }
  {  // attn_norm (h = residual + the previous layer's down partials, when it
     // left them) + q/k/v
    if (ws->down_pending > 1)
      FLOCK_TRY(act_image_reduce_enqueue(st, ws->h.as<float>(), ws->part.as<float>(),
                                         ws->down_pending, ws->h.as<float>(),
                                         L->w[W_ATTN_NORM]->data.as<float>(), c.eps, n, H, img));
    else
      FLOCK_TRY(act_image_enqueue(st, ws->h.as<float>(), H,
                                  L->w[W_ATTN_NORM]->data.as<float>(), c.eps, n, H, img));
    ws->down_pending = 0;
    TcArgs a = {};
    a.seg[0] = tc_seg_of(L->w[W_Q], ws->q.as<float>(), qw);
    a.seg[1] = tc_seg_of(L->w[W_K], ws->k.as<float>(), kvw);
    a.seg[2] = tc_seg_of(L->w[W_V], ws->v.as<float>(), kvw);
    a.nseg = 3;
    a.K = H;
    a.M = n;
    a.img = img;
    a.err = err;
    FLOCK_TRY(gemm_tc_enqueue(st, QT_Q8, EPI_STORE, a, d->sm_count, ws->part.bytes / 4));
  }
  FLOCK_TRY(enqueue_qk_attn(L, n, true, true));
  {  // o_proj + residual on h
    FLOCK_TRY(ws->atc_nz > 1 ? act_image_enqueue(st, nullptr, qw, nullptr, 0.0f, n, qw, img,
                                                 ws->atc_part.as<float>(), ws->atc_nz, c.n_heads)
                             : act_image_enqueue(st, ws->attn.as<float>(), qw, nullptr, 0.0f, n,
                                                 qw, img));
    TcArgs a = {};
    a.seg[0] = tc_seg_of(L->w[W_O], L->tp ? ws->tp_part.as<float>() : ws->h.as<float>(), H);
    a.nseg = 1;
    a.K = qw;
    a.M = n;
    a.img = img;
    a.res = ws->h.as<float>();
    a.res_stride = H;
    a.err = err;
    a.part = ws->part.as<float>();
    // a split-K o_proj leaves its partials for the ffn_norm image to sum
    FLOCK_TRY(gemm_tc_enqueue(st, QT_Q8, L->tp ? EPI_STORE : EPI_RESIDUAL, a, d->sm_count,
                              ws->part.bytes / 4, !L->tp));
    if (L->tp) FLOCK_TRY(tp_sum_into_h(L, n));
    o_split = L->tp ? 1 : a.ksplit;
  }
  {  // ffn_norm (h = residual + o_proj, when split) + gate | up
    if (o_split > 1)
      FLOCK_TRY(act_image_reduce_enqueue(st, ws->h.as<float>(), ws->part.as<float>(), o_split,
                                         ws->h.as<float>(),
                                         L->w[W_FFN_NORM]->data.as<float>(), c.eps, n, H, img));
    else
      FLOCK_TRY(act_image_enqueue(st, ws->h.as<float>(), H,
                                  L->w[W_FFN_NORM]->data.as<float>(), c.eps, n, H, img));
    TcArgs a = {};
    a.seg[0] = tc_seg_of(L->w[W_GATE], ws->gu.as<float>(), 2 * F);
    a.seg[1] = tc_seg_of(L->w[W_UP], ws->gu.as<float>() + F, 2 * F);
    a.nseg = 2;
    a.K = H;
    a.M = n;
    a.img = img;
    a.err = err;
    FLOCK_TRY(gemm_tc_enqueue(st, QT_Q8, EPI_STORE, a, d->sm_count, ws->part.bytes / 4));
  }
  {  // SwiGLU (in the image pass) + down + residual on h
    FLOCK_TRY(act_image_swiglu_enqueue(st, ws->gu.as<float>(), n, F, img));
    TcArgs a = {};
    a.seg[0] = tc_seg_of(L->w[W_DOWN], L->tp ? ws->tp_part.as<float>() : ws->h.as<float>(), H);
    a.nseg = 1;
    a.K = F;
    a.M = n;
    a.img = img;
    a.res = ws->h.as<float>();
    a.res_stride = H;
    a.err = err;
    a.part = ws->part.as<float>();
    // with a next layer in the same pass (ws->defer_down), a split-K down
    // leaves its partials for that layer's attn_norm image to sum
    const bool defer = !L->tp && ws->defer_down;
    FLOCK_TRY(gemm_tc_enqueue(st, QT_Q8, L->tp ? EPI_STORE : EPI_RESIDUAL, a, d->sm_count,
                              ws->part.bytes / 4, defer));
    if (defer && a.ksplit > 1) ws->down_pending = a.ksplit;
    if (L->tp) FLOCK_TRY(tp_sum_into_h(L, n));
  }
  return FLOCK_OK;
}

int ws_check_errors(Workspace* ws) {
  if (!ws->tc_err.p) return FLOCK_OK;
  int e = 0;
  FLOCK_CK(cudaMemcpy(&e, ws->tc_err.p, 4, cudaMemcpyDeviceToHost));
  if (e) {
    cudaMemset(ws->tc_err.p, 0, 4);
    set_error("tensor-core prefill GEMM gave up waiting (code %d)", e);
    return FLOCK_E_CUDA;
  }
  return FLOCK_OK;
}

int layer_enqueue(flock_layer* L, int n, bool advance, const PrefetchList& pf_next, bool pdl) {
  if (n > 1 && L->cfg.prefill == FLOCK_PREFILL_TENSOR) return layer_enqueue_tc(L, n, advance);
  flock_dev* d = L->dev;
  Workspace* ws = L->ws;
  const flock_layer_config& c = L->cfg;
  const int qw = c.n_heads * c.head_dim, kvw = c.n_kv_heads * c.head_dim;
  const float* g_attn = L->w[W_ATTN_NORM]->data.as<float>();
  const float* g_q = L->w[W_Q_NORM]->data.as<float>();
  const float* g_k = L->w[W_K_NORM]->data.as<float>();
  const float* g_ffn = L->w[W_FFN_NORM]->data.as<float>();

  // 1. attn_norm + q/k/v projections (one launch, three outputs)
  {
    GemvArgs a = {};
    a.seg[0] = seg_of(L->w[W_Q], ws->q.as<float>(), qw);
    a.seg[1] = seg_of(L->w[W_K], ws->k.as<float>(), kvw);
    a.seg[2] = seg_of(L->w[W_V], ws->v.as<float>(), kvw);
    a.nseg = 3;
    a.K = c.hidden;
    a.n_tokens = n;
    a.x = ws->h.as<float>();
    a.x_stride = c.hidden;
    a.norm_gain = g_attn;
    a.eps = c.eps;
    if (advance) {
      a.ctl = L->ctl;
      a.ctl_n = n;
    }
    pf_add(a.pf, L->w[W_O]);
    FLOCK_TRY(launch_gemv(d, QT_Q8, EPI_STORE, a, pdl));
  }
  // 2-3. q/k norm + RoPE + KV append, attention
  if (n == 1 && c.attention == FLOCK_ATTN_FAST) {
    AttnFastArgs a = {};
    a.q = ws->q.as<float>();
    a.k = ws->k.as<float>();
    a.v = ws->v.as<float>();
    a.q_norm = g_q;
    a.k_norm = g_k;
    a.inv_freq = L->inv_freq.as<float>();
    a.kcache = L->kcache.p;
    a.vcache = L->vcache.p;
    a.kv_bf16 = c.kv_dtype == FLOCK_KV_BF16;
    a.kv_fp8 = c.kv_dtype == FLOCK_KV_FP8;
    a.ctl = L->ctl;
    a.out = ws->attn.as<float>();
    a.part = ws->attn_part.as<float>();
    a.count = ws->attn_count.as<uint32_t>();
    a.n_heads = c.n_heads;
    a.n_kv_heads = c.n_kv_heads;
    a.head_dim = c.head_dim;
    a.splits = ws->attn_splits;
    a.eps = c.eps;
    a.neox = c.rope_pairing == FLOCK_ROPE_NEOX;
    a.chunk_cap = (c.max_keys + a.splits - 1) / a.splits;
    a.combine = 1;
    a.rope_cs = ws->rope.as<float2>();
    a.rope_rows = ws->rope_rows;
    a.max_keys = c.max_keys;
    pf_add(a.pf, L->w[W_GATE]);
    pf_add(a.pf, L->w[W_UP]);
    const size_t smem = attn_fast_smem(a.chunk_cap);
    // all shared memory: a long cache's splits run three 75 KB CTAs per SM
    auto kaf = c.kv_dtype == FLOCK_KV_FP8    ? k_attn_decode_fast<FLOCK_KV_FP8>
               : c.kv_dtype == FLOCK_KV_BF16 ? k_attn_decode_fast<FLOCK_KV_BF16>
                                             : k_attn_decode_fast<FLOCK_KV_F32>;
    FLOCK_TRY(kernel_setup((const void*)kaf, 200 * 1024, cudaSharedmemCarveoutMaxShared));
    FLOCK_CK(launch_ex(d->stream, kaf, dim3(c.n_kv_heads, a.splits),
                       dim3(ATTN_FAST_THREADS), smem, pdl, a));
  } else {
    FLOCK_TRY(enqueue_qk_attn(L, n, pdl, false));
  }
  // 4. o_proj + residual, in place on h (tensor parallel: a partial, summed
  // across ranks, then added)
  {
    GemvArgs a = {};
    const bool split = split_residual(L, n);
    a.seg[0] = seg_of(L->w[W_O], (L->tp || split) ? ws->tp_part.as<float>() : ws->h.as<float>(),
                      c.hidden);
    a.nseg = 1;
    a.K = qw;
    a.n_tokens = n;
    a.x = ws->attn.as<float>();
    a.x_stride = qw;
    a.res = ws->h.as<float>();
    a.res_stride = c.hidden;
    pf_add(a.pf, L->w[W_DOWN]);
    FLOCK_TRY(launch_gemv(d, QT_Q8, (L->tp || split) ? EPI_STORE : EPI_RESIDUAL, a, pdl));
    if (L->tp) FLOCK_TRY(tp_sum_into_h(L, n));
    if (split) FLOCK_TRY(add_split_residual(L, n));
  }
  // 5. ffn_norm + gate/up + SwiGLU
  {
    GemvArgs a = {};
    a.seg[0] = seg_of(L->w[W_GATE], ws->act.as<float>(), c.ffn);
    a.seg[1] = seg_of(L->w[W_UP], ws->act.as<float>(), c.ffn);
    a.nseg = 2;
    a.K = c.hidden;
    a.n_tokens = n;
    a.x = ws->h.as<float>();
    a.x_stride = c.hidden;
    a.norm_gain = g_ffn;
    a.eps = c.eps;
    a.pf = pf_next;
    FLOCK_TRY(launch_gemv(d, QT_Q8, EPI_SWIGLU, a, pdl));
  }
  // 6. down + residual, in place on h (tensor parallel as o_proj)
  {
    GemvArgs a = {};
    const bool split = split_residual(L, n);
    a.seg[0] = seg_of(L->w[W_DOWN], (L->tp || split) ? ws->tp_part.as<float>() : ws->h.as<float>(),
                      c.hidden);
    a.nseg = 1;
    a.K = c.ffn;
    a.n_tokens = n;
    a.x = ws->act.as<float>();
    a.x_stride = c.ffn;
    a.res = ws->h.as<float>();
    a.res_stride = c.hidden;
    FLOCK_TRY(launch_gemv(d, QT_Q8, (L->tp || split) ? EPI_STORE : EPI_RESIDUAL, a, pdl));
    if (L->tp) FLOCK_TRY(tp_sum_into_h(L, n));
    if (split) FLOCK_TRY(add_split_residual(L, n));
  }
  return FLOCK_OK;
}

}  // namespace flock

using namespace flock;

// ================================================================ C ABI

extern "C" {

const char* flock_last_error(void) { return g_err.c_str(); }
const char* flock_version(void) { return "flock_b200 0.1 sm_100a"; }

int flock_dev_open(int ordinal, flock_dev** out) {
  if (!out) return FLOCK_E_ARG;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    set_error("no CUDA device");
    return FLOCK_E_CUDA;
  }
  if (ordinal < 0 || ordinal >= n) {
    set_error("device %d out of range (%d devices)", ordinal, n);
    return FLOCK_E_ARG;
  }
  FLOCK_CK(cudaSetDevice(ordinal));
  cudaDeviceProp prop;
  FLOCK_CK(cudaGetDeviceProperties(&prop, ordinal));
  if (prop.major != 10) {
    set_error("device %d is sm_%d%d; this library is built for sm_100a (B200)", ordinal,
              prop.major, prop.minor);
    return FLOCK_E_UNSUPPORTED;
  }
  flock_dev* d = new flock_dev();
  d->ordinal = ordinal;
  d->sm_count = prop.multiProcessorCount;
  FLOCK_CK(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
  FLOCK_CK(cudaEventCreate(&d->t0));
  FLOCK_CK(cudaEventCreate(&d->t1));
  int rc;
  if ((rc = d->am_val.alloc(4096 * 4)) || (rc = d->am_idx.alloc(4096 * 4)) ||
      (rc = d->am_count.alloc(16)) || (rc = d->am_best_val.alloc(16)) ||
      (rc = d->am_best_idx.alloc(16))) {
    delete d;
    return rc;
  }
  FLOCK_CK(cudaMemset(d->am_count.p, 0, 16));
  *out = d;
  return FLOCK_OK;
}

int flock_dev_close(flock_dev* d) {
  flock::dev_release(d);
  return FLOCK_OK;
}

int flock_dev_sync(flock_dev* d) {
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

int flock_dev_sm_count(flock_dev* d, int* out) {
  *out = d->sm_count;
  return FLOCK_OK;
}

int flock_dev_timer_start(flock_dev* d) {
  FLOCK_CK(cudaEventRecord(d->t0, d->stream));
  return FLOCK_OK;
}

int flock_dev_timer_stop(flock_dev* d, float* ms) {
  FLOCK_CK(cudaEventRecord(d->t1, d->stream));
  FLOCK_CK(cudaEventSynchronize(d->t1));
  FLOCK_CK(cudaEventElapsedTime(ms, d->t0, d->t1));
  return FLOCK_OK;
}

// ---------------------------------------------------------------- repack

int flock_repack_q8(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* qs,
                    uint8_t* scales) {
  if (!packed || !qs || !scales || rows < 0 || cols % 32) {
    set_error("repack_q8: cols %lld must be a multiple of 32", (long long)cols);
    return FLOCK_E_ARG;
  }
  const int64_t nb = cols / 32;
  for (int64_t r = 0; r < rows; r++)
    for (int64_t b = 0; b < nb; b++) {
      const uint8_t* src = packed + (r * nb + b) * 34;
      scales[(r * nb + b) * 2] = src[0];
      scales[(r * nb + b) * 2 + 1] = src[1];
      memcpy(qs + r * cols + b * 32, src + 2, 32);
    }
  return FLOCK_OK;
}

int flock_repack_q4(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* qs,
                    uint8_t* scales) {
  if (!packed || !qs || !scales || rows < 0 || cols % 32) {
    set_error("repack_q4: cols %lld must be a multiple of 32", (long long)cols);
    return FLOCK_E_ARG;
  }
  const int64_t nb = cols / 32;
  for (int64_t r = 0; r < rows; r++)
    for (int64_t b = 0; b < nb; b++) {
      const uint8_t* src = packed + (r * nb + b) * 18;
      scales[(r * nb + b) * 2] = src[0];
      scales[(r * nb + b) * 2 + 1] = src[1];
      memcpy(qs + (r * nb + b) * 16, src + 2, 16);
    }
  return FLOCK_OK;
}

// --------------------------------------------------------------- tensors

int flock_tensor_from_split(flock_dev* dev, int dtype, const uint8_t* qs, const uint8_t* scales,
                            int64_t rows, int64_t cols, flock_tensor** out) {
  if (!dev || !qs || !scales || !out || rows < 1 || cols < 32 || cols % 32 ||
      (dtype != FLOCK_Q8_0 && dtype != FLOCK_Q4_0)) {
    set_error("tensor: bad split tensor %lldx%lld dtype %d", (long long)rows, (long long)cols,
              dtype);
    return FLOCK_E_ARG;
  }
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  flock_tensor* t = new flock_tensor();
  t->dev = flock::dev_retain(dev);
  t->dtype = dtype;
  t->rows = rows;
  t->cols = cols;
  const int64_t nb = cols / 32;
  t->sc_stride = (int)((nb + 7) / 8 * 8);
  const int64_t qs_bytes = dtype == FLOCK_Q8_0 ? rows * cols : rows * nb * 16;
  int rc;
  if ((rc = t->qs.alloc(qs_bytes)) || (rc = t->sc.alloc(rows * t->sc_stride * 2))) {
    flock_tensor_free(t);
    return rc;
  }
  cudaError_t e = cudaMemcpy(t->qs.p, qs, qs_bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    if (t->sc_stride == nb) {
      e = cudaMemcpy(t->sc.p, scales, rows * nb * 2, cudaMemcpyHostToDevice);
    } else {
      e = cudaMemset(t->sc.p, 0, t->sc.bytes);
      if (e == cudaSuccess)
        e = cudaMemcpy2D(t->sc.p, t->sc_stride * 2, scales, nb * 2, nb * 2, rows,
                         cudaMemcpyHostToDevice);
    }
  }
  if (e != cudaSuccess) {
    set_error("tensor upload failed: %s", cudaGetErrorString(e));
    flock_tensor_free(t);
    return FLOCK_E_CUDA;
  }
  *out = t;
  return FLOCK_OK;
}

int flock_tensor_from_packed(flock_dev* dev, int dtype, const uint8_t* packed, int64_t rows,
                             int64_t cols, flock_tensor** out) {
  if (!packed || cols % 32 || rows < 1) {
    set_error("tensor: cols %lld must be a multiple of 32", (long long)cols);
    return FLOCK_E_ARG;
  }
  const int64_t nb = cols / 32;
  std::vector<uint8_t> qs(dtype == FLOCK_Q8_0 ? rows * cols : rows * nb * 16);
  std::vector<uint8_t> sc(rows * nb * 2);
  int rc = dtype == FLOCK_Q8_0 ? flock_repack_q8(packed, rows, cols, qs.data(), sc.data())
                               : flock_repack_q4(packed, rows, cols, qs.data(), sc.data());
  if (rc) return rc;
  return flock_tensor_from_split(dev, dtype, qs.data(), sc.data(), rows, cols, out);
}

int flock_tensor_from_f32(flock_dev* dev, const float* data, int64_t n, flock_tensor** out) {
  if (!dev || !data || n < 1 || !out) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  flock_tensor* t = new flock_tensor();
  t->dev = flock::dev_retain(dev);
  t->dtype = FLOCK_F32;
  t->rows = 1;
  t->cols = n;
  int rc = t->data.alloc(n * 4);
  if (rc) {
    flock_tensor_free(t);
    return rc;
  }
  FLOCK_CK(cudaMemcpy(t->data.p, data, n * 4, cudaMemcpyHostToDevice));
  *out = t;
  return FLOCK_OK;
}

int flock_tensor_from_bytes(flock_dev* dev, const void* data, int64_t bytes, flock_tensor** out) {
  if (!dev || bytes < 1 || !out) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  const int64_t padded = (bytes + 3) & ~(int64_t)3;
  flock_tensor* t = new flock_tensor();
  t->dev = flock::dev_retain(dev);
  t->dtype = FLOCK_F32;
  t->rows = 1;
  t->cols = padded / 4;
  int rc = t->data.alloc(padded);
  if (rc) {
    flock_tensor_free(t);
    return rc;
  }
  FLOCK_CK(cudaMemset(t->data.p, 0, padded));
  if (data) FLOCK_CK(cudaMemcpy(t->data.p, data, bytes, cudaMemcpyHostToDevice));
  *out = t;
  return FLOCK_OK;
}

int flock_tensor_read(const flock_tensor* t, int64_t offset, int64_t bytes, void* out) {
  if (!t || !out || offset < 0 || bytes < 0) return FLOCK_E_ARG;
  if (t->dtype != FLOCK_F32) {
    set_error("readBack: only f32/raw tensors are readable (quantized planes stay on the device)");
    return FLOCK_E_ARG;
  }
  if (offset + bytes > (int64_t)t->data.bytes) {
    set_error("readBack: range [%lld, %lld) is outside the %lld-byte buffer", (long long)offset,
              (long long)(offset + bytes), (long long)t->data.bytes);
    return FLOCK_E_LIMIT;
  }
  if (!bytes) return FLOCK_OK;
  FLOCK_CK(cudaSetDevice(t->dev->ordinal));
  FLOCK_CK(cudaMemcpy(out, (const uint8_t*)t->data.p + offset, bytes, cudaMemcpyDeviceToHost));
  return FLOCK_OK;
}

int flock_tensor_free(flock_tensor* t) {
  if (t) {
    flock_dev* d = t->dev;
    if (d) cudaSetDevice(d->ordinal);
    delete t;
    flock::dev_release(d);
  }
  return FLOCK_OK;
}

int flock_tensor_bytes(const flock_tensor* t, int64_t* out) {
  *out = t->dtype == FLOCK_F32 ? (int64_t)t->data.bytes : (int64_t)(t->qs.bytes + t->sc.bytes);
  return FLOCK_OK;
}

// ------------------------------------------------------------ op level

}  // extern "C"

namespace {
struct Tmp {
  DBuf b;
  template <typename T>
  int put(const T* host, size_t n) {
    FLOCK_TRY(b.alloc(n * sizeof(T)));
    if (host) FLOCK_CK(cudaMemcpy(b.p, host, n * sizeof(T), cudaMemcpyHostToDevice));
    return FLOCK_OK;
  }
};
}  // namespace

extern "C" {

int flock_op_matvec(flock_dev* d, const flock_tensor* w, const float* x, int n_tokens,
                    float* out) {
  if (!d || !w || !x || !out || n_tokens < 1 || w->dtype == FLOCK_F32) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  Tmp tx, to;
  FLOCK_TRY(tx.put(x, (size_t)n_tokens * w->cols));
  FLOCK_TRY(to.put<float>(nullptr, (size_t)n_tokens * w->rows));
  GemvArgs a = {};
  a.seg[0] = seg_of(w, to.b.as<float>(), (int)w->rows);
  a.nseg = 1;
  a.K = (int)w->cols;
  a.n_tokens = n_tokens;
  a.x = tx.b.as<float>();
  a.x_stride = (int)w->cols;
  FLOCK_TRY(launch_gemv(d, w->dtype == FLOCK_Q8_0 ? QT_Q8 : QT_Q4, EPI_STORE, a, false));
  FLOCK_CK(cudaMemcpyAsync(out, to.b.p, (size_t)n_tokens * w->rows * 4, cudaMemcpyDeviceToHost,
                           d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

static int matvec_timed(flock_dev* d, const flock_tensor* w, int n_tokens, int iters, bool cold,
                        float* ms_per_call, bool fast = false) {
  if (!d || !w || n_tokens < 1 || iters < 1 || !ms_per_call || w->dtype == FLOCK_F32)
    return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  std::vector<float> hx((size_t)n_tokens * w->cols);
  uint32_t s = 12345u;
  for (auto& v : hx) {  // xorshift32 in [-1, 1)
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    v = (float)((double)s / 2147483648.0 - 1.0);
  }
  Tmp tx, to;
  FLOCK_TRY(tx.put(hx.data(), hx.size()));
  FLOCK_TRY(to.put<float>(nullptr, (size_t)n_tokens * w->rows));
  GemvArgs a = {};
  a.seg[0] = seg_of(w, to.b.as<float>(), (int)w->rows);
  a.nseg = 1;
  a.K = (int)w->cols;
  a.n_tokens = n_tokens;
  a.x = tx.b.as<float>();
  a.x_stride = (int)w->cols;
  const int qt = w->dtype == FLOCK_Q8_0 ? QT_Q8 : QT_Q4;
  auto go = [&](bool pdl) {
    return fast ? launch_gemv_fast(d, qt, EPI_STORE, a, pdl) : launch_gemv(d, qt, EPI_STORE, a, pdl);
  };
  FLOCK_TRY(go(false));  // warm-up
  if (!cold) {
    FLOCK_CK(cudaEventRecord(d->t0, d->stream));
    for (int i = 0; i < iters; i++) FLOCK_TRY(go(true));
    FLOCK_CK(cudaEventRecord(d->t1, d->stream));
    FLOCK_CK(cudaEventSynchronize(d->t1));
    float ms = 0;
    FLOCK_CK(cudaEventElapsedTime(&ms, d->t0, d->t1));
    *ms_per_call = ms / iters;
    return FLOCK_OK;
  }
  // cold: evict L2 with a 256 MiB write before each launch, time each alone
  DBuf flush;
  FLOCK_TRY(flush.alloc((size_t)256 << 20));
  float total = 0;
  for (int i = 0; i < iters; i++) {
    FLOCK_CK(cudaMemsetAsync(flush.p, i & 0xff, flush.bytes, d->stream));
    FLOCK_CK(cudaEventRecord(d->t0, d->stream));
    FLOCK_TRY(go(false));
    FLOCK_CK(cudaEventRecord(d->t1, d->stream));
    FLOCK_CK(cudaEventSynchronize(d->t1));
    float ms = 0;
    FLOCK_CK(cudaEventElapsedTime(&ms, d->t0, d->t1));
    total += ms;
  }
  *ms_per_call = total / iters;
  return FLOCK_OK;
}

int flock_op_matvec_timed(flock_dev* d, const flock_tensor* w, int n_tokens, int iters,
                          float* ms_per_call) {
  return matvec_timed(d, w, n_tokens, iters, false, ms_per_call);
}

int flock_op_matvec_timed_cold(flock_dev* d, const flock_tensor* w, int n_tokens, int iters,
                               float* ms_per_call) {
  return matvec_timed(d, w, n_tokens, iters, true, ms_per_call);
}

int flock_op_matvec_fast(flock_dev* d, const flock_tensor* w, const float* x, float* out) {
  if (!d || !w || !x || !out || w->dtype == FLOCK_F32) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  Tmp tx, to;
  FLOCK_TRY(tx.put(x, (size_t)w->cols));
  FLOCK_TRY(to.put<float>(nullptr, (size_t)w->rows));
  GemvArgs a = {};
  a.seg[0] = seg_of(w, to.b.as<float>(), (int)w->rows);
  a.nseg = 1;
  a.K = (int)w->cols;
  a.n_tokens = 1;
  a.x = tx.b.as<float>();
  a.x_stride = (int)w->cols;
  FLOCK_TRY(launch_gemv_fast(d, w->dtype == FLOCK_Q8_0 ? QT_Q8 : QT_Q4, EPI_STORE, a, false));
  FLOCK_CK(cudaMemcpyAsync(out, to.b.p, (size_t)w->rows * 4, cudaMemcpyDeviceToHost, d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

int flock_op_matvec_fast_timed(flock_dev* d, const flock_tensor* w, int iters, int cold,
                               float* ms_per_call) {
  return matvec_timed(d, w, 1, iters, cold != 0, ms_per_call, true);
}

int flock_op_rmsnorm(flock_dev* d, const float* x, const float* g, int n, int n_vecs, float eps,
                     float* out) {
  if (!d || !x || !g || !out || n < 1 || n_vecs < 1) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  Tmp tx, tg, to;
  FLOCK_TRY(tx.put(x, (size_t)n * n_vecs));
  FLOCK_TRY(tg.put(g, (size_t)n));
  FLOCK_TRY(to.put<float>(nullptr, (size_t)n * n_vecs));
  k_rmsnorm<<<n_vecs, 128, 0, d->stream>>>(tx.b.as<float>(), tg.b.as<float>(), to.b.as<float>(),
                                           n, n_vecs, eps);
  FLOCK_CK(cudaGetLastError());
  FLOCK_CK(cudaMemcpyAsync(out, to.b.p, (size_t)n * n_vecs * 4, cudaMemcpyDeviceToHost,
                           d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

}  // extern "C"

namespace flock {
// kernels/rope.wgsl:50: one thread per rotated pair, in place.
static __global__ void k_rope(float* x, const float* inv_freq, int n_tokens, int n_heads, int head_dim,
                       int pos0, int neox) {
  const int half = head_dim / 2;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (int64_t)n_tokens * n_heads * half) return;
  const int j = gid % half;
  const int head = (gid / half) % n_heads;
  const int tok = gid / ((int64_t)half * n_heads);
  const float theta = fmul((float)(pos0 + tok), inv_freq[j]);
  const float c = __double2float_rn(cos((double)theta));
  const float s = __double2float_rn(sin((double)theta));
  float* hb = x + ((int64_t)tok * n_heads + head) * head_dim;
  const int ia = neox ? j : 2 * j, ib = neox ? j + half : 2 * j + 1;
  const float a = hb[ia], b = hb[ib];
  hb[ia] = ffma(-b, s, fmul(a, c));
  hb[ib] = ffma(b, c, fmul(a, s));
}
}  // namespace flock

extern "C" {

int flock_op_rope(flock_dev* d, const float* x, int n_tokens, int n_heads, int head_dim,
                  int pos0, const float* inv_freq, int pairing, float* out) {
  if (!d || !x || !inv_freq || !out || head_dim % 2) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  const size_t n = (size_t)n_tokens * n_heads * head_dim;
  Tmp tx, ti;
  FLOCK_TRY(tx.put(x, n));
  FLOCK_TRY(ti.put(inv_freq, (size_t)head_dim / 2));
  const int64_t pairs = (int64_t)n_tokens * n_heads * (head_dim / 2);
  k_rope<<<(unsigned)((pairs + 63) / 64), 64, 0, d->stream>>>(
      tx.b.as<float>(), ti.b.as<float>(), n_tokens, n_heads, head_dim, pos0,
      pairing == FLOCK_ROPE_NEOX);
  FLOCK_CK(cudaGetLastError());
  FLOCK_CK(cudaMemcpyAsync(out, tx.b.p, n * 4, cudaMemcpyDeviceToHost, d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

static int ew_op(flock_dev* d, const float* a, const float* b, int64_t n, float* out, bool swiglu) {
  if (!d || !a || !b || !out || n < 1) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  Tmp ta, tb, to;
  FLOCK_TRY(ta.put(a, (size_t)n));
  FLOCK_TRY(tb.put(b, (size_t)n));
  FLOCK_TRY(to.put<float>(nullptr, (size_t)n));
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (swiglu)
    k_swiglu<<<blocks, 256, 0, d->stream>>>(ta.b.as<float>(), tb.b.as<float>(), to.b.as<float>(), n);
  else
    k_add<<<blocks, 256, 0, d->stream>>>(ta.b.as<float>(), tb.b.as<float>(), to.b.as<float>(), n);
  FLOCK_CK(cudaGetLastError());
  FLOCK_CK(cudaMemcpyAsync(out, to.b.p, n * 4, cudaMemcpyDeviceToHost, d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

int flock_op_swiglu(flock_dev* d, const float* g, const float* u, int64_t n, float* out) {
  return ew_op(d, g, u, n, out, true);
}

int flock_op_add(flock_dev* d, const float* a, const float* b, int64_t n, float* out) {
  return ew_op(d, a, b, n, out, false);
}

int flock_op_attention(flock_dev* d, const float* q, const float* k, const float* v, int n_heads,
                       int n_kv_heads, int head_dim, int n_keys, int mode, float* out) {
  if (!d || !q || !k || !v || !out || head_dim != 128 || n_keys < 1 || n_kv_heads < 1 ||
      n_heads % n_kv_heads) {
    set_error("attention: head_dim must be 128 and n_heads a multiple of n_kv_heads");
    return FLOCK_E_ARG;
  }
  FLOCK_CK(cudaSetDevice(d->ordinal));
  const size_t kvn = (size_t)n_keys * n_kv_heads * head_dim;
  Tmp tq, tk, tv, to, tc;
  FLOCK_TRY(tq.put(q, (size_t)n_heads * head_dim));
  FLOCK_TRY(tk.put(k, kvn));
  FLOCK_TRY(tv.put(v, kvn));
  FLOCK_TRY(to.put<float>(nullptr, (size_t)n_heads * head_dim));
  int ctl[2] = {n_keys - 1, 0};
  FLOCK_TRY(tc.put(ctl, 2));
  if (mode == FLOCK_ATTN_EXACT) {
    if ((size_t)n_keys * 4 > 200 * 1024) {
      set_error("exact attention: %d keys exceed the on-chip score buffer", n_keys);
      return FLOCK_E_UNSUPPORTED;
    }
    AttnArgs aa = {};
    aa.q = tq.b.as<float>();
    aa.kcache = tk.b.as<float>();
    aa.vcache = tv.b.as<float>();
    aa.out = to.b.as<float>();
    aa.ctl = tc.b.as<int>();
    aa.n_tokens = 1;
    aa.n_heads = n_heads;
    aa.n_kv_heads = n_kv_heads;
    aa.head_dim = head_dim;
    FLOCK_CK(cudaFuncSetAttribute(k_attn_decode_exact, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  200 * 1024));
    k_attn_decode_exact<<<n_heads, 256, (size_t)n_keys * 4, d->stream>>>(aa);
    FLOCK_CK(cudaGetLastError());
  } else {
    // split-K core on already-final q/k (the layer path fuses norm + RoPE)
    if (n_heads / n_kv_heads > 4) return FLOCK_E_UNSUPPORTED;
    Tmp tp, tcount;
    const int splits = 16;
    FLOCK_TRY(tp.put<float>(nullptr, (size_t)n_heads * splits * (head_dim + 2)));
    FLOCK_TRY(tcount.put<uint32_t>(nullptr, (size_t)n_kv_heads));
    FLOCK_CK(cudaMemset(tcount.b.p, 0, tcount.b.bytes));
    AttnFastArgs a = {};
    a.q = tq.b.as<float>();
    a.kcache = tk.b.p;
    a.vcache = tv.b.p;
    a.ctl = tc.b.as<int>();
    a.out = to.b.as<float>();
    a.part = tp.b.as<float>();
    a.count = tcount.b.as<uint32_t>();
    a.n_heads = n_heads;
    a.n_kv_heads = n_kv_heads;
    a.head_dim = head_dim;
    a.splits = splits;
    a.chunk_cap = (n_keys + splits - 1) / splits;
    a.combine = 1;
    const size_t smem = attn_fast_smem(a.chunk_cap);
    if (smem > 200 * 1024) return FLOCK_E_UNSUPPORTED;
    FLOCK_CK(cudaFuncSetAttribute(k_attn_decode_fast<FLOCK_KV_F32>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    k_attn_decode_fast<FLOCK_KV_F32>
        <<<dim3(n_kv_heads, splits), ATTN_FAST_THREADS, smem, d->stream>>>(a);
    FLOCK_CK(cudaGetLastError());
  }
  FLOCK_CK(cudaMemcpyAsync(out, to.b.p, (size_t)n_heads * head_dim * 4, cudaMemcpyDeviceToHost,
                           d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

int flock_op_attention_prefill(flock_dev* d, const float* q, const float* k, const float* v,
                               int n_heads, int n_kv_heads, int head_dim, int n_queries, int pos0,
                               float* out) {
  if (!d || !q || !k || !v || !out || head_dim != 128 || n_queries < 1 || pos0 < 0 ||
      n_kv_heads < 1 || n_heads % n_kv_heads) {
    set_error("attention_prefill: head_dim must be 128");
    return FLOCK_E_ARG;
  }
  FLOCK_CK(cudaSetDevice(d->ordinal));
  const int n_keys = pos0 + n_queries;
  const size_t kvn = (size_t)n_keys * n_kv_heads * head_dim;
  const size_t qn = (size_t)n_queries * n_heads * head_dim;
  Tmp tq, tk, tv, to, tc;
  FLOCK_TRY(tq.put(q, qn));
  FLOCK_TRY(tk.put(k, kvn));
  FLOCK_TRY(tv.put(v, kvn));
  FLOCK_TRY(to.put<float>(nullptr, qn));
  int ctl[2] = {pos0, 0};
  FLOCK_TRY(tc.put(ctl, 2));
  AttnArgs aa = {};
  aa.q = tq.b.as<float>();
  aa.kcache = tk.b.as<float>();
  aa.vcache = tv.b.as<float>();
  aa.out = to.b.as<float>();
  aa.ctl = tc.b.as<int>();
  aa.n_tokens = n_queries;
  aa.n_heads = n_heads;
  aa.n_kv_heads = n_kv_heads;
  aa.head_dim = head_dim;
  k_attn_prefill_exact<<<dim3(n_heads, n_queries), 128, 0, d->stream>>>(aa);
  FLOCK_CK(cudaGetLastError());
  FLOCK_CK(cudaMemcpyAsync(out, to.b.p, qn * 4, cudaMemcpyDeviceToHost, d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

int flock_op_embed(flock_dev* d, const flock_tensor* table, const int32_t* ids, int n,
                   float* out) {
  if (!d || !table || !ids || !out || n < 1 || table->dtype != FLOCK_Q8_0) return FLOCK_E_ARG;
  for (int i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= table->rows) {
      set_error("embed: id %d out of range 0..%lld", ids[i], (long long)table->rows - 1);
      return FLOCK_E_ARG;
    }
  FLOCK_CK(cudaSetDevice(d->ordinal));
  Tmp ti, to;
  FLOCK_TRY(ti.put(ids, (size_t)n));
  FLOCK_TRY(to.put<float>(nullptr, (size_t)n * table->cols));
  EmbedArgs a = {};
  a.qs = table->qs.as<uint8_t>();
  a.sc = table->sc.as<uint16_t>();
  a.ids = ti.b.as<int32_t>();
  a.out = to.b.as<float>();
  a.n_tokens = n;
  a.hidden = (int)table->cols;
  a.sc_stride = table->sc_stride;
  a.vocab = (int)table->rows;
  k_embed<<<n, 256, 0, d->stream>>>(a);
  FLOCK_CK(cudaGetLastError());
  FLOCK_CK(cudaMemcpyAsync(out, to.b.p, (size_t)n * table->cols * 4, cudaMemcpyDeviceToHost,
                           d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

int flock_op_argmax(flock_dev* d, const float* x, int64_t n, int64_t* index, float* value) {
  if (!d || !x || n < 1 || !index) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  Tmp tx;
  FLOCK_TRY(tx.put(x, (size_t)n));
  int blocks = (int)((n + 255) / 256);
  if (blocks > 2 * d->sm_count) blocks = 2 * d->sm_count;
  k_argmax<<<blocks, 256, 0, d->stream>>>(tx.b.as<float>(), n, d->am_val.as<float>(),
                                          d->am_idx.as<uint32_t>(), d->am_count.as<uint32_t>(),
                                          d->am_best_val.as<float>(), d->am_best_idx.as<int32_t>(),
                                          0);
  FLOCK_CK(cudaGetLastError());
  int32_t idx = 0;
  float val = 0;
  FLOCK_CK(cudaMemcpyAsync(&idx, d->am_best_idx.p, 4, cudaMemcpyDeviceToHost, d->stream));
  FLOCK_CK(cudaMemcpyAsync(&val, d->am_best_val.p, 4, cudaMemcpyDeviceToHost, d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  *index = (int64_t)(uint32_t)idx;
  if (value) *value = val;
  return FLOCK_OK;
}

// ------------------------------------------------------------------ layer

}  // extern "C"

namespace flock {
// Layer.fromBuffers (layer.ts:228) body: bind tensors by name, check the
// required set (requireWeights, :269) and shapes, allocate the KV cache.
// ws / ctl == nullptr -> the layer owns its workspace / position block.
int layer_build(flock_dev* dev, const flock_layer_config* cfg, int n_tensors,
                const char* const* names, flock_tensor* const* tensors, Workspace* ws,
                int* ctl, flock_layer** out) {
  if (!dev || !cfg || !names || !tensors || !out) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  flock_layer* L = new flock_layer();
  for (int i = 0; i < n_tensors; i++) {
    int slot = -1;
    for (int s = 0; s < W_COUNT; s++)
      if (names[i] && strcmp(names[i], kTensorNames[s]) == 0) slot = s;
    if (slot < 0) continue;  // extra tensors are ignored, as the reference ignores them
    const flock_tensor* t = tensors[i];
    const bool is_norm = slot >= W_ATTN_NORM;
    if (!t || (is_norm ? t->dtype != FLOCK_F32 : t->dtype != FLOCK_Q8_0)) {
      set_error("%s: neither a split Q8_0 tensor nor f32 data", names[i]);
      delete L;
      return FLOCK_E_ARG;
    }
    L->w[slot] = t;
  }
  std::string missing;
  int n_missing = 0;
  for (int s = 0; s < W_COUNT; s++)
    if (!L->w[s]) {
      missing += (n_missing ? ", " : "");
      missing += kTensorNames[s];
      n_missing++;
    }
  if (n_missing) {
    set_error("layer is missing %d tensor(s): %s", n_missing, missing.c_str());
    delete L;
    return FLOCK_E_MISSING;
  }
  // shapes
  const int qw = cfg->n_heads * cfg->head_dim, kvw = cfg->n_kv_heads * cfg->head_dim;
  struct { int s; int64_t r, c; } want[] = {
      {W_Q, qw, cfg->hidden},         {W_K, kvw, cfg->hidden},        {W_V, kvw, cfg->hidden},
      {W_O, cfg->hidden, qw},         {W_GATE, cfg->ffn, cfg->hidden}, {W_UP, cfg->ffn, cfg->hidden},
      {W_DOWN, cfg->hidden, cfg->ffn}};
  for (auto& w : want)
    if (L->w[w.s]->rows != w.r || L->w[w.s]->cols != w.c) {
      set_error("%s is %lldx%lld, config wants %lldx%lld", kTensorNames[w.s],
                (long long)L->w[w.s]->rows, (long long)L->w[w.s]->cols, (long long)w.r,
                (long long)w.c);
      delete L;
      return FLOCK_E_ARG;
    }
  int rc = layer_init(L, dev, *cfg, ws, ctl);
  if (rc) {
    flock_layer_free(L);
    return rc;
  }
  *out = L;
  return FLOCK_OK;
}
}  // namespace flock

extern "C" {

int flock_layer_create(flock_dev* dev, const flock_layer_config* cfg, int n_tensors,
                       const char* const* names, flock_tensor* const* tensors,
                       flock_layer** out) {
  return layer_build(dev, cfg, n_tensors, names, tensors, nullptr, nullptr, out);
}


int flock_layer_free(flock_layer* L) {
  if (L) {
    flock_dev* d = L->dev;
    if (d) {
      cudaSetDevice(d->ordinal);
      cudaStreamSynchronize(d->stream);
    }
    delete L;
    flock::dev_release(d);
  }
  return FLOCK_OK;
}

int flock_layer_encode(flock_layer* L, const float* hidden, int n) {
  if (!L) return FLOCK_E_ARG;
  const flock_layer_config& c = L->cfg;
  if (n < 1) {
    set_error("nTokens must be >= 1, got %d", n);
    return FLOCK_E_ARG;
  }
  if (n > c.max_prefill) {
    set_error("prefill of %d exceeds maxPrefill %d; chunk it", n, c.max_prefill);
    return FLOCK_E_STATE;
  }
  if (L->n_keys + n > c.max_keys) {
    if (n == 1) set_error("KV cache full at %d keys", c.max_keys);
    else set_error("KV cache would exceed %d keys (%d + %d)", c.max_keys, L->n_keys, n);
    return FLOCK_E_STATE;
  }
  FLOCK_CK(cudaSetDevice(L->dev->ordinal));
  if (hidden)
    FLOCK_CK(cudaMemcpyAsync(L->ws->h.p, hidden, (size_t)n * c.hidden * 4, cudaMemcpyHostToDevice,
                             L->dev->stream));
  PrefetchList none = {};
  FLOCK_TRY(layer_enqueue(L, n, true, none, true));
  L->n_keys += n;
  return FLOCK_OK;
}

int flock_layer_read_output(flock_layer* L, int n, float* out) {
  if (!L || !out || n < 1 || n > L->cfg.max_prefill) return FLOCK_E_ARG;
  FLOCK_CK(cudaMemcpyAsync(out, L->ws->h.p, (size_t)n * L->cfg.hidden * 4, cudaMemcpyDeviceToHost,
                           L->dev->stream));
  FLOCK_CK(cudaStreamSynchronize(L->dev->stream));
  return ws_check_errors(L->ws);
}

int flock_layer_rewind(flock_layer* L, int n_keys) {
  if (!L || n_keys < 0 || n_keys > L->cfg.max_keys) return FLOCK_E_ARG;
  int ctl[2] = {n_keys, 0};
  FLOCK_CK(cudaMemcpyAsync(L->ctl, ctl, sizeof ctl, cudaMemcpyHostToDevice, L->dev->stream));
  FLOCK_CK(cudaStreamSynchronize(L->dev->stream));
  L->n_keys = n_keys;
  return FLOCK_OK;
}

int flock_layer_reset(flock_layer* L) { return flock_layer_rewind(L, 0); }

int flock_layer_n_keys(const flock_layer* L, int* out) {
  *out = L->n_keys;
  return FLOCK_OK;
}

// OCP E4M3FN on the host: code -> value (exact), and value -> the nearest
// code (ties to even, magnitudes past 448 saturating to 448, NaN to 0x7F),
// the conversion the device's cvt.rn.satfinite performs.
static float host_fp8_value(uint8_t b) {
  const int sgn = b >> 7, e = (b >> 3) & 15, m = b & 7;
  if (e == 15 && m == 7) return NAN;
  const float mag = e == 0 ? std::ldexp((float)m, -9) : std::ldexp((float)(8 + m), e - 10);
  return sgn ? -mag : mag;
}
static uint8_t host_fp8_bits(float x) {
  if (std::isnan(x)) return 0x7F;
  const uint8_t sgn = std::signbit(x) ? 0x80 : 0;
  float a = std::fabs(x);
  if (a >= 448.0f) return sgn | 0x7E;
  int e2 = 0;
  std::frexp(a, &e2);            // a = f * 2^e2, f in [0.5, 1)
  int E = e2 - 1;                // a in [2^E, 2^(E+1))
  if (E < -6) E = -6;            // subnormals: steps of 2^-9
  const float step = std::ldexp(1.0f, E - 3);
  const float q = std::nearbyint(a / step);  // ties to even (the default rounding mode)
  const float r = q * step;
  if (r == 0.0f) return sgn;
  int re = 0;
  std::frexp(r, &re);
  const int Er = re - 1;
  if (Er < -6) return sgn | (uint8_t)(r / std::ldexp(1.0f, -9));  // subnormal code
  const int mant = (int)(r / std::ldexp(1.0f, Er - 3)) - 8;
  return sgn | (uint8_t)((Er + 7) << 3) | (uint8_t)mant;
}

int flock_layer_read_cache(flock_layer* L, float* k, float* v) {
  if (!L || !k || !v) return FLOCK_E_ARG;
  const size_t count = (size_t)L->n_keys * L->cfg.n_kv_heads * L->cfg.head_dim;
  if (count && L->cfg.kv_dtype == FLOCK_KV_FP8) {
    // e4m3 -> f32 exactly
    std::vector<uint8_t> kb(count), vb(count);
    FLOCK_CK(cudaMemcpyAsync(kb.data(), L->kcache.p, count, cudaMemcpyDeviceToHost,
                             L->dev->stream));
    FLOCK_CK(cudaMemcpyAsync(vb.data(), L->vcache.p, count, cudaMemcpyDeviceToHost,
                             L->dev->stream));
    FLOCK_CK(cudaStreamSynchronize(L->dev->stream));
    for (size_t i = 0; i < count; i++) {
      k[i] = host_fp8_value(kb[i]);
      v[i] = host_fp8_value(vb[i]);
    }
  } else if (count && L->cfg.kv_dtype == FLOCK_KV_BF16) {
    // bf16 -> f32 exactly: the stored bits become the high half
    std::vector<uint16_t> kb(count), vb(count);
    FLOCK_CK(cudaMemcpyAsync(kb.data(), L->kcache.p, count * 2, cudaMemcpyDeviceToHost,
                             L->dev->stream));
    FLOCK_CK(cudaMemcpyAsync(vb.data(), L->vcache.p, count * 2, cudaMemcpyDeviceToHost,
                             L->dev->stream));
    FLOCK_CK(cudaStreamSynchronize(L->dev->stream));
    for (size_t i = 0; i < count; i++) {
      const uint32_t kw = (uint32_t)kb[i] << 16, vw = (uint32_t)vb[i] << 16;
      memcpy(k + i, &kw, 4);
      memcpy(v + i, &vw, 4);
    }
  } else if (count) {
    FLOCK_CK(cudaMemcpyAsync(k, L->kcache.p, count * 4, cudaMemcpyDeviceToHost, L->dev->stream));
    FLOCK_CK(cudaMemcpyAsync(v, L->vcache.p, count * 4, cudaMemcpyDeviceToHost, L->dev->stream));
  }
  FLOCK_CK(cudaStreamSynchronize(L->dev->stream));
  return ws_check_errors(L->ws);
}

// f32 -> bf16 bits, rounded to nearest with ties to even (NaN stays a quiet NaN).
static uint16_t host_bf16_bits(float x) {
  uint32_t w;
  memcpy(&w, &x, 4);
  if ((w & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((w >> 16) | 0x40u);
  return (uint16_t)((w + 0x7fffu + ((w >> 16) & 1u)) >> 16);
}

int flock_layer_write_cache(flock_layer* L, const float* k, const float* v, int n_keys) {
  if (!L || !k || !v || n_keys < 0 || L->n_keys + n_keys > L->cfg.max_keys) return FLOCK_E_ARG;
  const size_t elems = (size_t)L->cfg.n_kv_heads * L->cfg.head_dim;
  const size_t row = elems * kv_elem_bytes(L->cfg);
  if (L->cfg.kv_dtype == FLOCK_KV_FP8) {
    const size_t count = elems * (size_t)n_keys;
    std::vector<uint8_t> kb(count), vb(count);
    for (size_t i = 0; i < count; i++) {
      kb[i] = host_fp8_bits(k[i]);
      vb[i] = host_fp8_bits(v[i]);
    }
    FLOCK_CK(cudaMemcpyAsync(L->kcache.as<uint8_t>() + L->n_keys * row, kb.data(), n_keys * row,
                             cudaMemcpyHostToDevice, L->dev->stream));
    FLOCK_CK(cudaMemcpyAsync(L->vcache.as<uint8_t>() + L->n_keys * row, vb.data(), n_keys * row,
                             cudaMemcpyHostToDevice, L->dev->stream));
    FLOCK_CK(cudaStreamSynchronize(L->dev->stream));  // before the host copies go
  } else if (L->cfg.kv_dtype == FLOCK_KV_BF16) {
    const size_t count = elems * (size_t)n_keys;
    std::vector<uint16_t> kb(count), vb(count);
    for (size_t i = 0; i < count; i++) {
      kb[i] = host_bf16_bits(k[i]);
      vb[i] = host_bf16_bits(v[i]);
    }
    FLOCK_CK(cudaMemcpyAsync(L->kcache.as<uint8_t>() + L->n_keys * row, kb.data(), n_keys * row,
                             cudaMemcpyHostToDevice, L->dev->stream));
    FLOCK_CK(cudaMemcpyAsync(L->vcache.as<uint8_t>() + L->n_keys * row, vb.data(), n_keys * row,
                             cudaMemcpyHostToDevice, L->dev->stream));
    FLOCK_CK(cudaStreamSynchronize(L->dev->stream));  // before the host copies go
  } else {
    FLOCK_CK(cudaMemcpyAsync(L->kcache.as<uint8_t>() + L->n_keys * row, k, n_keys * row,
                             cudaMemcpyHostToDevice, L->dev->stream));
    FLOCK_CK(cudaMemcpyAsync(L->vcache.as<uint8_t>() + L->n_keys * row, v, n_keys * row,
                             cudaMemcpyHostToDevice, L->dev->stream));
  }
  return flock_layer_rewind(L, L->n_keys + n_keys);
}

int flock_range_forward(flock_layer* const* layers, int n_layers, const float* x, int seq,
                        int offset, int reset, float* out) {
  if (!layers || n_layers < 1 || !x || !out || seq < 1) return FLOCK_E_ARG;
  for (int i = 0; i < n_layers; i++) {
    if (!layers[i] || layers[i]->dev != layers[0]->dev ||
        layers[i]->cfg.hidden != layers[0]->cfg.hidden) {
      set_error("range_forward: layers must share one device and hidden size");
      return FLOCK_E_ARG;
    }
    if (reset) FLOCK_TRY(flock_layer_reset(layers[i]));
    if (layers[i]->n_keys != offset) {
      set_error("offset %d does not match this cache's position %d", offset, layers[i]->n_keys);
      return FLOCK_E_STATE;
    }
  }
  flock_dev* d = layers[0]->dev;
  const size_t bytes = (size_t)seq * layers[0]->cfg.hidden * 4;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  FLOCK_TRY(flock_layer_encode(layers[0], x, seq));
  for (int i = 1; i < n_layers; i++) {
    // chain on the device: previous output -> this layer's input buffer
    if (layers[i]->ws != layers[i - 1]->ws)
      FLOCK_CK(cudaMemcpyAsync(layers[i]->ws->h.p, layers[i - 1]->ws->h.p, bytes,
                               cudaMemcpyDeviceToDevice, d->stream));
    FLOCK_TRY(flock_layer_encode(layers[i], nullptr, seq));
  }
  return flock_layer_read_output(layers[n_layers - 1], seq, out);
}

}  // extern "C"
