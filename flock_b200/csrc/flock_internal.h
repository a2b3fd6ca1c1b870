// Internal host-side structures of libflock_cuda.so (not part of the ABI).
#pragma once
#include <cuda_runtime.h>

#include <utility>

#include <atomic>

#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/flock_cuda.h"
#include "gemv.cuh"

namespace flock {

void set_error(const char* fmt, ...);

// Per (kernel, current device), once: when max_dyn_smem > 0, opt in to that
// much dynamic shared memory (the attribute is per device, so a process
// driving several GPUs needs it on each).
// Opt `func` in to max_dyn_smem bytes of dynamic shared memory (once per
// device); carveout >= 0 also sets its preferred shared-memory carveout (%).
int kernel_setup(const void* func, int max_dyn_smem, int carveout = -1);

// Device references (see flock_dev): retain returns its argument.
flock_dev* dev_retain(flock_dev* d);
void dev_release(flock_dev* d);

#define FLOCK_CK(call)                                                              \
  do {                                                                              \
    cudaError_t e_ = (call);                                                        \
    if (e_ != cudaSuccess) {                                                        \
      ::flock::set_error("CUDA error %s at %s:%d (%s)", cudaGetErrorString(e_),     \
                         __FILE__, __LINE__, #call);                                \
      return FLOCK_E_CUDA;                                                          \
    }                                                                               \
  } while (0)

#define FLOCK_TRY(expr)        \
  do {                         \
    int rc_ = (expr);          \
    if (rc_ != FLOCK_OK) return rc_; \
  } while (0)

// A device allocation owned by its holder.
struct DBuf {
  void* p = nullptr;
  size_t bytes = 0;
  int alloc(size_t n);
  void release();
  template <typename T>
  T* as() const { return reinterpret_cast<T*>(p); }
  ~DBuf() { release(); }
  DBuf() = default;
  DBuf(const DBuf&) = delete;
  DBuf& operator=(const DBuf&) = delete;
};

}  // namespace flock

// Every object created on a device (tensor, layer, model, shard, head,
// communicator) holds a reference, so flock_dev_close only drops the
// caller's reference and the device lives until the last object is freed.
struct flock_dev {
  std::atomic<int> refs{1};
  int ordinal = 0;
  int sm_count = 148;
  cudaStream_t stream = nullptr;
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  // scratch for op-level calls and argmax partials
  flock::DBuf am_val, am_idx, am_count, am_best_val, am_best_idx;
};

struct flock_tensor {
  flock_dev* dev = nullptr;
  int dtype = 0;
  int64_t rows = 0, cols = 0;
  int sc_stride = 0;  // f16 scales per row, padded to a multiple of 8
  flock::DBuf qs, sc, data;
};

struct flock_comm;

namespace flock {

// Activation buffers one layer step needs; a Model shares one across layers.
struct Workspace {
  int P = 0, H = 0, nH = 0, nKV = 0, hd = 0, F = 0;
  DBuf h, q, k, v, qn, attn, act;
  DBuf attn_part, attn_count;  // fast decode attention partials
  int attn_splits = 16;         // splits (attn_max_splits); partial slots per query head
  DBuf img, gu, tc_err, part;   // tensor-core prefill: activation image, gate|up rows, error word,
                                // split-K partials
  DBuf rope;                    // RoPE (cos, sin) [rope_rows][hd / 2] (k_rope_table)
  int rope_rows = 0;
  DBuf kv_img;                  // tensor-core prefill: f16 K / V^T tiles of the cache
  DBuf atc_part;                // tensor-core prefill attention: per key range O, m, l
  DBuf q_img;                   // tensor-core prefill: f16 rotated queries [nH][q_tiles][128 x 128]
  int q_tiles = 0;
  int atc_nz = 1;               // key ranges of the last tensor-core attention launch
  // tensor-core prefill across the layers of one pass: the enqueuer sets
  // defer_down when another layer follows, and down_pending is the number of
  // split-K partials of h in `part` that the next layer's first image sums
  bool defer_down = false;
  int down_pending = 0;
  DBuf tp_part, tp_all;         // tensor parallel: this rank's partial [P][H], all ranks
  DBuf wire;                    // FLK1 frames: the f16 payload on the device
  // tp_ranks >= 1 (a tensor-parallel model, one rank included): also the
  // partial / all-gather buffers; 0 = no tensor parallelism
  int alloc(const flock_layer_config& c, int sm_count, int tp_ranks = 0);
};

enum { W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN, W_ATTN_NORM, W_Q_NORM, W_K_NORM, W_FFN_NORM,
       W_COUNT };
extern const char* const kTensorNames[W_COUNT];

// Launch plan pieces
int launch_gemv(flock_dev* d, int QT, int EPI, const GemvArgs& a, bool pdl);
// FLOCK_MATVEC_FAST: one token per CTA row on the int8 tensor cores
// (store, residual and argmax epilogues; Q4_0 store only)
int launch_gemv_fast(flock_dev* d, int QT, int EPI, const GemvArgs& a, bool pdl);
// tensor-core prefill GEMM (flock_gemm.cu)
struct TcArgs;
struct TcSeg;
struct PeerXchg;
size_t act_image_bytes(int M, int K);
// A kernel launch on `st`; with `pdl` the launch may begin while the
// previous kernel of the stream still runs (programmatic dependent launch):
// the kernel must call griddepcontrol.wait before it touches anything that
// kernel writes or reads.
template <typename... KArgs, typename... Args>
static cudaError_t launch_ex(cudaStream_t st, void (*k)(KArgs...), dim3 grid, dim3 block,
                             size_t smem, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

int act_image_enqueue(cudaStream_t st, const float* x, int x_stride, const float* gain, float eps,
                      int M, int K, uint8_t* img, const float* atc_part = nullptr, int atc_nz = 0,
                      int n_heads = 0);
// The activation image of x = res + the split-K partials [red_nz][M][K]
// (summed as k_splitk_reduce sums them; x is also written to x_out), or of
// the SwiGLU of [gate | up] rows [M][2K] -- the reduce and SwiGLU kernels
// folded into the image pass.
int act_image_reduce_enqueue(cudaStream_t st, const float* res, const float* red_part, int red_nz,
                             float* x_out, const float* gain, float eps, int M, int K,
                             uint8_t* img);
int act_image_swiglu_enqueue(cudaStream_t st, const float* gu, int M, int K, uint8_t* img);
int gemm_tc_enqueue(cudaStream_t st, int qt, int epi, TcArgs& a, int sm_count,
                    size_t part_floats, bool defer_reduce = false);
TcSeg tc_seg_of(const flock_tensor* t, float* out, int out_stride);
// tensor-core prefill's device error word: FLOCK_E_CUDA (and cleared) if a tensor-core
// GEMM gave up waiting since the last check; call after a synchronisation.
int ws_check_errors(Workspace* ws);
int gemv_grid(flock_dev* d, int total_groups);

}  // namespace flock

struct flock_layer {
  flock_dev* dev = nullptr;
  flock_layer_config cfg{};
  const flock_tensor* w[flock::W_COUNT] = {};
  flock::DBuf kcache, vcache, ctl_own, inv_freq;
  int* ctl = nullptr;          // {pos, n_last} on the device (own or the model's)
  int n_keys = 0;              // host mirror
  // tensor parallel: this layer is one rank's slice; o_proj and down give
  // partial sums that are all-gathered over `tp` and added in rank order
  flock_comm* tp = nullptr;
  int tp_n = 1;
  flock::PeerXchg* xchg = nullptr;  // decode steps: the fused peer exchange (else NCCL)
  flock::Workspace* ws = nullptr;
  flock::Workspace ws_own;     // standalone layers own their workspace
  bool owns_ws = false;
};

namespace flock {
// Bytes per cached key/value element: 4 (FLOCK_KV_F32) or 2 (FLOCK_KV_BF16).
inline size_t kv_elem_bytes(const flock_layer_config& c) {
  return c.kv_dtype == FLOCK_KV_BF16 ? 2 : c.kv_dtype == FLOCK_KV_FP8 ? 1 : 4;
}
// Enqueue one layer step over ws->h (in place): n tokens at the layer's pos.
// `advance` = this launch advances the layer's ctl; pf_next = L2 prefetch
// hint for whatever follows the layer (may be empty).
int layer_enqueue(flock_layer* L, int n, bool advance, const PrefetchList& pf_next, bool pdl);
int layer_init(flock_layer* L, flock_dev* dev, const flock_layer_config& cfg, Workspace* ws,
               int* shared_ctl);
int comm_send(flock_comm* c, const void* p, size_t n_f32, int peer);
int comm_recv(flock_comm* c, void* p, size_t n_f32, int peer);
int comm_wait(flock_comm* c);
// NCCL all-gather of `bytes` per rank between device buffers on the
// communicator's stream (out is [n_ranks][bytes], rank order).
int comm_allgather_dev(flock_comm* c, const void* in, void* out, size_t bytes);
// Fused peer-memory exchange (flock_peer.cu): h[i] += sum over ranks of the
// ranks' part[i], rank order; `cap` floats per exchange.  init and free are
// collectives over the communicator.
int peer_xchg_init(flock_comm* c, int64_t cap, PeerXchg** out);
int peer_xchg_run(PeerXchg* x, cudaStream_t st, float* h, const float* part, int64_t n);
int peer_xchg_check(PeerXchg* x);
int peer_xchg_free(PeerXchg* x);
int comm_rank(const flock_comm* c, int* rank, int* n_ranks);
flock_dev* comm_device(const flock_comm* c);
int layer_build(flock_dev* dev, const flock_layer_config* cfg, int n_tensors,
                const char* const* names, flock_tensor* const* tensors, Workspace* ws, int* ctl,
                flock_layer** out);
}  // namespace flock
