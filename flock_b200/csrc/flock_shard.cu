// Tensor parallelism (kernels/shard.ts, shard_ref.ts, q8_shard.wgsl,
// shard_reduce.wgsl) and the NCCL communicator for multi-GPU runs.
//
// ShardedMatvec / ShardedHead keep the reference's single-device form --
// N shards of one tensor on one GPU, each its own sliced allocation -- which
// is what makes the split testable against the unsharded kernel.  The
// multi-GPU forms are the same shards, one per rank, with the partial-sum
// reduction (input-split) done by NCCL all-reduce and the head's argmax by
// an 8-byte all-gather of (value, index) pairs (shard_ref.ts:437 rule).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "flock_internal.h"
#include "gemv.cuh"

using namespace flock;

namespace flock {

// shard_ref.ts:97 shardRanges
static int shard_ranges(int64_t total, int n, int64_t align, std::vector<int64_t>& start,
                        std::vector<int64_t>& count) {
  if (n < 1) {
    set_error("n shards must be >= 1, got %d", n);
    return FLOCK_E_ARG;
  }
  if (total < 0 || align < 1) {
    set_error("total must be >= 0 and align >= 1");
    return FLOCK_E_ARG;
  }
  if (total % align) {
    set_error("total %lld is not a multiple of align %lld", (long long)total, (long long)align);
    return FLOCK_E_ARG;
  }
  const int64_t units = total / align;
  if (units < n) {
    set_error("cannot cut %lld into %d shards aligned to %lld: only %lld units", (long long)total,
              n, (long long)align, (long long)units);
    return FLOCK_E_ARG;
  }
  start.resize(n);
  count.resize(n);
  int64_t at = 0;
  for (int i = 0; i < n; i++) {
    count[i] = (units / n + (i < units % n ? 1 : 0)) * align;
    start[i] = at;
    at += count[i];
  }
  return FLOCK_OK;
}

// shard_reduce.wgsl:47: serial sum in shard order (the order is the contract).
static __global__ void k_shard_reduce(const float* parts, int n_shards, int64_t n, float* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = parts[i];
  for (int s = 1; s < n_shards; s++) acc = __fadd_rn(acc, parts[(int64_t)s * n + i]);
  out[i] = acc;
}

static __global__ void k_argmax_plain(const float* x, int64_t n, float* pval, uint32_t* pidx) {
  // one CTA: lowest index among the maxima of x[0..n)
  __shared__ float wv[32];
  __shared__ uint32_t wi[32];
  float bv = -FLT_MAX;
  uint32_t bi = 0xFFFFFFFFu;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    if (v > bv || (v == bv && (uint32_t)i < bi)) {
      bv = v;
      bi = (uint32_t)i;
    }
  }
  for (int s = 16; s > 0; s >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, bv, s);
    const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, s);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    wv[threadIdx.x >> 5] = bv;
    wi[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (wv[w] > bv || (wv[w] == bv && wi[w] < bi)) {
        bv = wv[w];
        bi = wi[w];
      }
    *pval = bv;
    *pidx = bi;
  }
}

}  // namespace flock

struct flock_shard {
  flock_dev* dev = nullptr;
  int64_t rows = 0, cols = 0;
  int n = 0, dir = 0;
  std::vector<int64_t> start, count;
  std::vector<flock_tensor*> shards;
  DBuf x, out, parts;
};

struct flock_head {
  flock_dev* dev = nullptr;
  int64_t vocab = 0, hidden = 0;
  int n = 0;
  std::vector<int64_t> start, count;
  std::vector<flock_tensor*> shards;
  DBuf x, logits, sval, sidx;
  std::vector<float> last_val;
  std::vector<int64_t> last_idx;
};

static int upload_slice(flock_dev* dev, const uint8_t* qs, const uint8_t* sc, int64_t rows,
                        int64_t cols, int64_t r0, int64_t r1, int64_t c0, int64_t c1,
                        flock_tensor** out) {
  const int64_t nb = cols / 32, w = c1 - c0, wb = w / 32, b0 = c0 / 32, nr = r1 - r0;
  std::vector<uint8_t> q((size_t)(nr * w)), s((size_t)(nr * wb * 2));
  for (int64_t r = 0; r < nr; r++) {  // shard_ref.ts:137 sliceRows / :166 sliceCols
    memcpy(q.data() + r * w, qs + (r0 + r) * cols + c0, (size_t)w);
    memcpy(s.data() + r * wb * 2, sc + ((r0 + r) * nb + b0) * 2, (size_t)(wb * 2));
  }
  return flock_tensor_from_split(dev, FLOCK_Q8_0, q.data(), s.data(), nr, w, out);
}

static int run_gemv_rows(flock_dev* d, const flock_tensor* t, const float* x, float* out) {
  GemvArgs a = {};
  a.seg[0].qs = t->qs.as<uint8_t>();
  a.seg[0].sc = t->sc.as<uint16_t>();
  a.seg[0].out = out;
  a.seg[0].rows = (int)t->rows;
  a.seg[0].sc_stride = t->sc_stride;
  a.seg[0].out_stride = (int)t->rows;
  a.nseg = 1;
  a.K = (int)t->cols;
  a.n_tokens = 1;
  a.x = x;
  a.x_stride = (int)t->cols;
  return launch_gemv(d, QT_Q8, EPI_STORE, a, false);
}

extern "C" {

int flock_shard_matvec_create(flock_dev* dev, const uint8_t* qs, const uint8_t* scales,
                              int64_t rows, int64_t cols, int n, int direction,
                              int64_t binding_limit, flock_shard** out) {
  if (!dev || !qs || !scales || !out || rows < 1 || cols < 32) return FLOCK_E_ARG;
  if (cols % 32) {
    set_error("cols %lld must be a multiple of 32", (long long)cols);
    return FLOCK_E_ARG;
  }
  if (direction != 0 && direction != 1) return FLOCK_E_ARG;
  std::vector<int64_t> st, ct;
  FLOCK_TRY(shard_ranges(direction == 0 ? rows : cols, n, direction == 0 ? 1 : 32, st, ct));
  if (binding_limit > 0) {  // shard.ts:229-243 capacity check before any upload
    int64_t mx = 0;
    for (int i = 0; i < n; i++) {
      const int64_t r = direction == 0 ? ct[i] : rows, c = direction == 0 ? cols : ct[i];
      const int64_t b = std::max(r * c, r * ((c + 31) / 32) * 2);
      mx = std::max(mx, b);
    }
    if (mx > binding_limit) {
      set_error("%s-wise %d shards of %lldx%lld need a %lld byte binding, over the %lld byte limit",
                direction == 0 ? "row" : "col", n, (long long)rows, (long long)cols,
                (long long)mx, (long long)binding_limit);
      return FLOCK_E_LIMIT;
    }
  }
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  flock_shard* s = new flock_shard();
  s->dev = flock::dev_retain(dev);
  s->rows = rows;
  s->cols = cols;
  s->n = n;
  s->dir = direction;
  s->start = st;
  s->count = ct;
  int rc = FLOCK_OK;
  for (int i = 0; i < n && !rc; i++) {
    flock_tensor* t = nullptr;
    rc = direction == 0 ? upload_slice(dev, qs, scales, rows, cols, st[i], st[i] + ct[i], 0, cols, &t)
                        : upload_slice(dev, qs, scales, rows, cols, 0, rows, st[i], st[i] + ct[i], &t);
    if (!rc) s->shards.push_back(t);
  }
  if (!rc) rc = s->x.alloc(cols * 4);
  if (!rc) rc = s->out.alloc(rows * 4);
  if (!rc && direction == 1) rc = s->parts.alloc((size_t)n * rows * 4);
  if (rc) {
    flock_shard_matvec_free(s);
    return rc;
  }
  *out = s;
  return FLOCK_OK;
}

int flock_shard_matvec_free(flock_shard* s) {
  if (!s) return FLOCK_OK;
  for (auto* t : s->shards) flock_tensor_free(t);
  flock_dev* d = s->dev;
  delete s;
  flock::dev_release(d);
  return FLOCK_OK;
}

int flock_shard_matvec_run(flock_shard* s, const float* x, float* y) {
  if (!s || !x || !y) return FLOCK_E_ARG;
  flock_dev* d = s->dev;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  FLOCK_CK(cudaMemcpyAsync(s->x.p, x, s->cols * 4, cudaMemcpyHostToDevice, d->stream));
  for (int i = 0; i < s->n; i++) {
    if (s->dir == 0) {
      FLOCK_TRY(run_gemv_rows(d, s->shards[i], s->x.as<float>(), s->out.as<float>() + s->start[i]));
    } else {
      FLOCK_TRY(run_gemv_rows(d, s->shards[i], s->x.as<float>() + s->start[i],
                              s->parts.as<float>() + (size_t)i * s->rows));
    }
  }
  if (s->dir == 1) {
    k_shard_reduce<<<(unsigned)((s->rows + 255) / 256), 256, 0, d->stream>>>(
        s->parts.as<float>(), s->n, s->rows, s->out.as<float>());
    FLOCK_CK(cudaGetLastError());
  }
  FLOCK_CK(cudaMemcpyAsync(y, s->out.p, s->rows * 4, cudaMemcpyDeviceToHost, d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  return FLOCK_OK;
}

int flock_shard_matvec_partials(flock_shard* s, float* parts) {
  if (!s || !parts) return FLOCK_E_ARG;
  if (s->dir != 1) {
    set_error("row-wise sharding has no partials buffer");
    return FLOCK_E_STATE;
  }
  FLOCK_CK(cudaMemcpyAsync(parts, s->parts.p, (size_t)s->n * s->rows * 4, cudaMemcpyDeviceToHost,
                           s->dev->stream));
  FLOCK_CK(cudaStreamSynchronize(s->dev->stream));
  return FLOCK_OK;
}

int flock_shard_matvec_wire_bytes(const flock_shard* s, int64_t* out) {
  // shard.ts:411: row-wise broadcasts x (cols floats) to each shard;
  // column-wise moves each shard's full-length partial (rows floats).
  *out = s->dir == 0 ? (int64_t)s->n * s->cols * 4 : (int64_t)s->n * s->rows * 4;
  return FLOCK_OK;
}

int flock_sharded_head_create(flock_dev* dev, const uint8_t* qs, const uint8_t* scales,
                              int64_t vocab, int64_t hidden, int n, flock_head** out) {
  if (!dev || !qs || !scales || !out || vocab < 1 || hidden % 32) return FLOCK_E_ARG;
  std::vector<int64_t> st, ct;
  FLOCK_TRY(shard_ranges(vocab, n, 1, st, ct));
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  flock_head* h = new flock_head();
  h->dev = flock::dev_retain(dev);
  h->vocab = vocab;
  h->hidden = hidden;
  h->n = n;
  h->start = st;
  h->count = ct;
  int rc = FLOCK_OK;
  for (int i = 0; i < n && !rc; i++) {
    flock_tensor* t = nullptr;
    rc = upload_slice(dev, qs, scales, vocab, hidden, st[i], st[i] + ct[i], 0, hidden, &t);
    if (!rc) h->shards.push_back(t);
  }
  if (!rc) rc = h->x.alloc(hidden * 4);
  if (!rc) rc = h->logits.alloc(vocab * 4);
  if (!rc) rc = h->sval.alloc((size_t)n * 4);
  if (!rc) rc = h->sidx.alloc((size_t)n * 4);
  if (rc) {
    flock_sharded_head_free(h);
    return rc;
  }
  *out = h;
  return FLOCK_OK;
}

int flock_sharded_head_free(flock_head* h) {
  if (!h) return FLOCK_OK;
  for (auto* t : h->shards) flock_tensor_free(t);
  flock_dev* d = h->dev;
  delete h;
  flock::dev_release(d);
  return FLOCK_OK;
}

int flock_sharded_head_run(flock_head* h, const float* x, float* logits, int32_t* token) {
  if (!h || !x) return FLOCK_E_ARG;
  flock_dev* d = h->dev;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  FLOCK_CK(cudaMemcpyAsync(h->x.p, x, h->hidden * 4, cudaMemcpyHostToDevice, d->stream));
  for (int i = 0; i < h->n; i++) {
    float* lg = h->logits.as<float>() + h->start[i];
    FLOCK_TRY(run_gemv_rows(d, h->shards[i], h->x.as<float>(), lg));
    // per-shard argmax.wgsl pass1+pass2: (value, shard-local index)
    k_argmax_plain<<<1, 1024, 0, d->stream>>>(lg, h->count[i], h->sval.as<float>() + i,
                                             h->sidx.as<uint32_t>() + i);
    FLOCK_CK(cudaGetLastError());
  }
  std::vector<float> v(h->n);
  std::vector<uint32_t> ix(h->n);
  FLOCK_CK(cudaMemcpyAsync(v.data(), h->sval.p, h->n * 4, cudaMemcpyDeviceToHost, d->stream));
  FLOCK_CK(cudaMemcpyAsync(ix.data(), h->sidx.p, h->n * 4, cudaMemcpyDeviceToHost, d->stream));
  if (logits)
    FLOCK_CK(cudaMemcpyAsync(logits, h->logits.p, h->vocab * 4, cudaMemcpyDeviceToHost, d->stream));
  FLOCK_CK(cudaStreamSynchronize(d->stream));
  // shard_ref.ts:437 reduceShardArgmax: global index = rowOffset + index,
  // strictly greater or equal-with-lower-index wins.
  int64_t bi = -1;
  float bv = -INFINITY;
  h->last_val.assign(v.begin(), v.end());
  h->last_idx.resize(h->n);
  for (int i = 0; i < h->n; i++) {
    h->last_idx[i] = ix[i];
    const int64_t gi = h->start[i] + (int64_t)ix[i];
    if (v[i] > bv || (v[i] == bv && gi < bi)) {
      bv = v[i];
      bi = gi;
    }
  }
  if (token) *token = (int32_t)bi;
  return FLOCK_OK;
}

int flock_sharded_head_shard_argmax(flock_head* h, float* values, int64_t* index,
                                    int64_t* row_offset) {
  if (!h || h->last_val.empty()) {
    set_error("run the head first");
    return FLOCK_E_STATE;
  }
  for (int i = 0; i < h->n; i++) {
    values[i] = h->last_val[i];
    index[i] = h->last_idx[i];
    row_offset[i] = h->start[i];
  }
  return FLOCK_OK;
}

}  // extern "C"

// ====================================================================== NCCL

namespace {
struct Nccl {
  void* so = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool load() {
    if (so) return true;
    so = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!so) {
      set_error("NCCL (libnccl.so.2) could not be loaded: %s", dlerror());
      return false;
    }
#define SYM(f) f = reinterpret_cast<decltype(f)>(dlsym(so, "nccl" #f))
    SYM(GetUniqueId);
    SYM(CommInitRankConfig);
    SYM(CommDestroy);
    SYM(CommAbort);
    SYM(CommGetAsyncError);
    SYM(Send);
    SYM(Recv);
    SYM(AllReduce);
    SYM(AllGather);
    SYM(GetErrorString);
#undef SYM
    if (!GetUniqueId || !CommInitRankConfig || !Send || !Recv || !AllReduce || !AllGather ||
        !CommGetAsyncError || !CommAbort || !CommDestroy || !GetErrorString) {
      set_error("libnccl.so.2 lacks required symbols");
      return false;
    }
    return true;
  }
} g_nccl;
}  // namespace

struct flock_comm {
  flock_dev* dev = nullptr;
  ncclComm_t comm = nullptr;
  int n_ranks = 0, rank = 0, timeout_ms = 30000;
  DBuf tmp_in, tmp_out;
};

namespace flock {
// Wait for the communicator's stream with a deadline; abort the communicator
// if NCCL reports an error or the deadline passes (no unbounded host wait).
int comm_wait(flock_comm* c) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q = cudaStreamQuery(c->dev->stream);
    if (q == cudaSuccess) return FLOCK_OK;
    if (q != cudaErrorNotReady) {
      set_error("CUDA error during collective: %s", cudaGetErrorString(q));
      return FLOCK_E_CUDA;
    }
    ncclResult_t ae = ncclSuccess;
    if (g_nccl.CommGetAsyncError) g_nccl.CommGetAsyncError(c->comm, &ae);
    if (ae != ncclSuccess && ae != ncclInProgress) {
      set_error("NCCL async error: %s", g_nccl.GetErrorString ? g_nccl.GetErrorString(ae) : "?");
      if (g_nccl.CommAbort) g_nccl.CommAbort(c->comm);
      c->comm = nullptr;
      return FLOCK_E_NCCL;
    }
    const double ms = std::chrono::duration<double, std::milli>(
                          std::chrono::steady_clock::now() - t0).count();
    if (ms > c->timeout_ms) {
      set_error("collective timed out after %d ms (a peer rank is gone?)", c->timeout_ms);
      if (g_nccl.CommAbort) g_nccl.CommAbort(c->comm);
      c->comm = nullptr;
      return FLOCK_E_NCCL;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}
}  // namespace flock

#define NCCL_CK(call)                                                                  \
  do {                                                                                 \
    ncclResult_t r_ = (call);                                                          \
    if (r_ != ncclSuccess && r_ != ncclInProgress) {                                   \
      set_error("NCCL error %s at %s", g_nccl.GetErrorString(r_), #call);             \
      return FLOCK_E_NCCL;                                                             \
    }                                                                                  \
  } while (0)

// A communicator created non-blocking may answer an enqueue with
// ncclInProgress; it takes the next call only once ncclCommGetAsyncError
// reports ncclSuccess.  Bounded by the communicator's timeout (then aborted).
static int nccl_settle(flock_comm* c, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return FLOCK_OK;
  if (r != ncclInProgress) {
    set_error("NCCL error %s at %s", g_nccl.GetErrorString(r), what);
    return FLOCK_E_NCCL;
  }
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclInProgress;
    g_nccl.CommGetAsyncError(c->comm, &st);
    if (st == ncclSuccess) return FLOCK_OK;
    if (st != ncclInProgress) {
      set_error("NCCL error %s after %s", g_nccl.GetErrorString(st), what);
      g_nccl.CommAbort(c->comm);
      c->comm = nullptr;
      return FLOCK_E_NCCL;
    }
    if (std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count() >
        c->timeout_ms) {
      set_error("%s still in progress after %d ms (a peer rank is gone?)", what, c->timeout_ms);
      g_nccl.CommAbort(c->comm);
      c->comm = nullptr;
      return FLOCK_E_NCCL;
    }
    std::this_thread::yield();
  }
}
#define NCCL_ISSUE(c, call) FLOCK_TRY(nccl_settle((c), (call), #call))

extern "C" {

int flock_comm_unique_id(uint8_t id_out[128]) {
  if (!g_nccl.load()) return FLOCK_E_NCCL;
  ncclUniqueId id;
  NCCL_CK(g_nccl.GetUniqueId(&id));
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  memcpy(id_out, &id, 128);
  return FLOCK_OK;
}

int flock_comm_init(flock_dev* dev, int n_ranks, int rank, const uint8_t id[128], int timeout_ms,
                    flock_comm** out) {
  if (!dev || !id || !out || n_ranks < 1 || rank < 0 || rank >= n_ranks) return FLOCK_E_ARG;
  if (!g_nccl.load()) return FLOCK_E_NCCL;
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  flock_comm* c = new flock_comm();
  c->dev = flock::dev_retain(dev);
  c->n_ranks = n_ranks;
  c->rank = rank;
  c->timeout_ms = timeout_ms > 0 ? timeout_ms : 30000;
  ncclUniqueId uid;
  memcpy(&uid, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // non-blocking init so a missing peer times out here
  ncclResult_t r = g_nccl.CommInitRankConfig(&c->comm, n_ranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    set_error("ncclCommInitRankConfig: %s", g_nccl.GetErrorString(r));
    flock_dev* d = c->dev;
    delete c;
    flock::dev_release(d);
    return FLOCK_E_NCCL;
  }
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclInProgress;
    g_nccl.CommGetAsyncError(c->comm, &st);
    if (st == ncclSuccess) break;
    if (st != ncclInProgress) {
      set_error("NCCL init failed: %s", g_nccl.GetErrorString(st));
      g_nccl.CommAbort(c->comm);
      flock_dev* d = c->dev;
      delete c;
      flock::dev_release(d);
      return FLOCK_E_NCCL;
    }
    if (std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count() >
        c->timeout_ms) {
      set_error("NCCL init timed out after %d ms", c->timeout_ms);
      g_nccl.CommAbort(c->comm);
      flock_dev* d = c->dev;
      delete c;
      flock::dev_release(d);
      return FLOCK_E_NCCL;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  *out = c;
  return FLOCK_OK;
}

int flock_comm_free(flock_comm* c) {
  if (!c) return FLOCK_OK;
  if (c->comm) {
    cudaStreamSynchronize(c->dev->stream);
    g_nccl.CommDestroy(c->comm);
  }
  flock_dev* d = c->dev;
  delete c;
  flock::dev_release(d);
  return FLOCK_OK;
}

int flock_comm_allreduce_f32(flock_comm* c, const float* in, float* out, int64_t n) {
  if (!c || !c->comm || !in || !out || n < 1) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(c->dev->ordinal));
  FLOCK_TRY(c->tmp_in.alloc(n * 4));
  FLOCK_TRY(c->tmp_out.alloc(n * 4));
  FLOCK_CK(cudaMemcpyAsync(c->tmp_in.p, in, n * 4, cudaMemcpyHostToDevice, c->dev->stream));
  NCCL_ISSUE(c, g_nccl.AllReduce(c->tmp_in.p, c->tmp_out.p, (size_t)n, ncclFloat32, ncclSum, c->comm,
                           c->dev->stream));
  FLOCK_CK(cudaMemcpyAsync(out, c->tmp_out.p, n * 4, cudaMemcpyDeviceToHost, c->dev->stream));
  return comm_wait(c);
}

int flock_comm_allgather_bytes(flock_comm* c, const void* in, void* out, int64_t bytes) {
  if (!c || !c->comm || !in || !out || bytes < 1) return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(c->dev->ordinal));
  FLOCK_TRY(c->tmp_in.alloc(bytes));
  FLOCK_TRY(c->tmp_out.alloc(bytes * c->n_ranks));
  FLOCK_CK(cudaMemcpyAsync(c->tmp_in.p, in, bytes, cudaMemcpyHostToDevice, c->dev->stream));
  NCCL_ISSUE(c, g_nccl.AllGather(c->tmp_in.p, c->tmp_out.p, (size_t)bytes, ncclUint8, c->comm,
                           c->dev->stream));
  FLOCK_CK(cudaMemcpyAsync(out, c->tmp_out.p, bytes * c->n_ranks, cudaMemcpyDeviceToHost,
                           c->dev->stream));
  return comm_wait(c);
}

}  // extern "C"

// The hidden-state hops of the layer pipeline live with the model (they need
// its workspace); see flock_model.cu.
namespace flock {
int comm_allgather_dev(flock_comm* c, const void* in, void* out, size_t bytes) {
  if (!c->comm) return FLOCK_E_NCCL;
  NCCL_ISSUE(c, g_nccl.AllGather(in, out, bytes, ncclUint8, c->comm, c->dev->stream));
  return FLOCK_OK;
}
int comm_send(flock_comm* c, const void* p, size_t n_f32, int peer) {
  if (!c->comm) return FLOCK_E_NCCL;
  NCCL_ISSUE(c, g_nccl.Send(p, n_f32, ncclFloat32, peer, c->comm, c->dev->stream));
  return FLOCK_OK;
}
flock_dev* comm_device(const flock_comm* c) { return c->dev; }
int comm_rank(const flock_comm* c, int* rank, int* n_ranks) {
  *rank = c->rank;
  *n_ranks = c->n_ranks;
  return c->comm ? FLOCK_OK : FLOCK_E_NCCL;
}
int comm_recv(flock_comm* c, void* p, size_t n_f32, int peer) {
  if (!c->comm) return FLOCK_E_NCCL;
  NCCL_ISSUE(c, g_nccl.Recv(p, n_f32, ncclFloat32, peer, c->comm, c->dev->stream));
  return FLOCK_OK;
}
}  // namespace flock
