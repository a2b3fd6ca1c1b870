// Fused peer-memory exchange for tensor-parallel decode: the o_proj / down
// partials of every rank summed in rank order, without NCCL.
//
// Each rank exports one buffer and one flag array (cudaIpcGetMemHandle) and
// maps every peer's (cudaIpcOpenMemHandle, NVLink).  One exchange is one
// kernel on each rank:
//   1. push: write this rank's partial [n] into slot [parity][rank] of every
//      rank's buffer (plain stores over NVLink; no TMA, no multicast);
//   2. publish: system-scope fence, then a release store of the exchange's
//      epoch into flag [parity][rank] of every rank;
//   3. wait: acquire-poll this rank's own flags until every rank has
//      published this epoch (bounded by the global timer: a peer that never
//      arrives sets the error word and the kernel returns);
//   4. reduce: h += p_0 + p_1 + ... + p_{N-1} summed serially in rank order
//      (shard_ref.ts:327 shardReduceRef's order), the arithmetic of the NCCL
//      path's k_tp_reduce_residual, so both paths give identical bits.
// Two parity slots: a rank can run at most one exchange ahead of a peer (its
// next exchange needs that peer's next partial, which the peer publishes only
// after it has reduced the current one), so the slot it writes is never the
// one the peer is still reading.
#include <cuda_runtime.h>

#include <vector>

#include "flock_internal.h"
#include "mbar.cuh"

namespace flock {

struct PeerXchg {
  flock_comm* comm = nullptr;
  int rank = 0, n = 1;
  int64_t cap = 0;                 // floats per (slot, rank)
  float* buf = nullptr;            // this rank's [2][n][cap]
  uint32_t* flag = nullptr;        // this rank's [2][n][XCHG_MAX_CTAS]
  std::vector<void*> opened;       // peers' mapped buffers / flags (closed at free)
  float** d_bufs = nullptr;        // [n] device pointers (own or mapped)
  uint32_t** d_flags = nullptr;    // [n]
  uint32_t* epoch = nullptr;       // exchanges completed, per exchange CTA
  int* err = nullptr;              // 3 = a peer never published (sticky: never cleared)
  uint64_t wait_ns = WAIT_NS;      // how long a CTA waits for the peers' flags
  bool failed = false;             // a wait ran out: every later exchange is refused
};

namespace {

FLOCK_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
FLOCK_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// CTA c exchanges elements [c * XCHG_CHUNK, (c + 1) * XCHG_CHUNK): four per
// thread as one 128-bit load / store, its own flag and epoch slots, so CTAs
// need not run at the same time.
constexpr int XCHG_THREADS = 256, XCHG_CHUNK = 4 * XCHG_THREADS, XCHG_MAX_CTAS = 16;

__global__ void __launch_bounds__(XCHG_THREADS) k_peer_xchg(const float* __restrict__ part,
                                                            float* h, int n, int rank,
                                                            int n_ranks, int64_t cap,
                                                            float* const* bufs,
                                                            uint32_t* const* flags,
                                                            uint32_t* epochs, int* err,
                                                            uint64_t wait_ns) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  const int t = threadIdx.x, c = blockIdx.x;
  const int i = c * XCHG_CHUNK + 4 * t;  // n is a multiple of 4
  if (t == 0) {
    s_epoch = epochs[c] + 1u;
    // after a timeout this rank's epochs no longer match its peers': stop
    // exchanging for good (graph replays included) rather than sum partials
    // of another step
    s_ok = *(volatile int*)err == 0;
  }
  __syncthreads();
  if (!s_ok) return;
  const uint32_t e = s_epoch, slot = e & 1u;
  const bool mine = i < n;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (mine) v = *reinterpret_cast<const float4*>(part + i);
  if (n_ranks == 1) {  // nothing to exchange: the one partial is the sum
    if (mine) {
      float4 hv = *reinterpret_cast<float4*>(h + i);
      hv = make_float4(fadd(hv.x, v.x), fadd(hv.y, v.y), fadd(hv.z, v.z), fadd(hv.w, v.w));
      *reinterpret_cast<float4*>(h + i) = hv;
    }
    if (t == 0) epochs[c] = e;
    return;
  }
  if (mine)
    for (int r = 0; r < n_ranks; r++)
      *reinterpret_cast<float4*>(bufs[r] + ((int64_t)slot * n_ranks + rank) * cap + i) = v;
  // the CTA barrier orders every thread's pushes before thread 0's release
  // stores, and a release is cumulative: one system-scope release per flag
  // publishes the whole CTA's data
  __syncthreads();
  if (t == 0) {
    const int fo = (int)(slot * n_ranks + rank) * XCHG_MAX_CTAS + c;
    for (int r = 0; r < n_ranks; r++) st_release_sys(flags[r] + fo, e);
    const uint32_t* own = flags[rank] + (int)slot * n_ranks * XCHG_MAX_CTAS + c;
    int ok = 1;
    uint64_t t0 = 0;
    for (int r = 0; r < n_ranks && ok; r++) {
      for (uint32_t k = 0; (int32_t)(ld_acquire_sys(own + r * XCHG_MAX_CTAS) - e) < 0; k++) {
        if ((k & 63) != 63) continue;
        const uint64_t now = globaltimer_ns();
        if (!t0) t0 = now;
        if (now - t0 > wait_ns || k >= WAIT_MAX_POLLS) {
          atomicExch(err, 3);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  if (mine) {
    const float* own = bufs[rank] + (int64_t)slot * n_ranks * cap + i;
    float4 acc = __ldcg(reinterpret_cast<const float4*>(own));
    for (int r = 1; r < n_ranks; r++) {
      const float4 p = __ldcg(reinterpret_cast<const float4*>(own + (int64_t)r * cap));
      acc = make_float4(fadd(acc.x, p.x), fadd(acc.y, p.y), fadd(acc.z, p.z), fadd(acc.w, p.w));
    }
    float4 hv = *reinterpret_cast<float4*>(h + i);
    hv = make_float4(fadd(hv.x, acc.x), fadd(hv.y, acc.y), fadd(hv.z, acc.z), fadd(hv.w, acc.w));
    *reinterpret_cast<float4*>(h + i) = hv;
  }
  if (t == 0) epochs[c] = e;
}

}  // namespace

int peer_xchg_free(PeerXchg* x) {
  if (!x) return FLOCK_OK;
  // every rank must be done with every buffer before any is released
  if (x->comm && x->n > 1) {
    float one = 1.0f, sum = 0.0f;
    flock_comm_allreduce_f32(x->comm, &one, &sum, 1);
  }
  for (void* p : x->opened) cudaIpcCloseMemHandle(p);
  cudaFree(x->buf);
  cudaFree(x->flag);
  cudaFree(x->d_bufs);
  cudaFree(x->d_flags);
  cudaFree(x->epoch);
  cudaFree(x->err);
  delete x;
  return FLOCK_OK;
}

int peer_xchg_init(flock_comm* c, int64_t cap, PeerXchg** out) {
  *out = nullptr;
  int rank = 0, n = 1;
  FLOCK_TRY(comm_rank(c, &rank, &n));
  flock_dev* dev = comm_device(c);
  FLOCK_CK(cudaSetDevice(dev->ordinal));
  PeerXchg* x = new PeerXchg();
  x->comm = c;
  x->rank = rank;
  x->n = n;
  x->cap = cap;
  auto fail = [&](int rc) {
    peer_xchg_free(x);
    return rc;
  };
  if (cudaMalloc(&x->buf, (size_t)2 * n * cap * 4) != cudaSuccess ||
      cudaMalloc(&x->flag, (size_t)2 * n * 16 * 4) != cudaSuccess ||
      cudaMalloc(&x->d_bufs, (size_t)n * sizeof(float*)) != cudaSuccess ||
      cudaMalloc(&x->d_flags, (size_t)n * sizeof(uint32_t*)) != cudaSuccess ||
      cudaMalloc(&x->epoch, 16 * 4) != cudaSuccess || cudaMalloc(&x->err, 16) != cudaSuccess) {
    set_error("peer exchange: device allocation failed");
    x->comm = nullptr;  // no collective on this path: the peers may not have got here
    return fail(FLOCK_E_NOMEM);
  }
  if (cudaMemset(x->flag, 0, (size_t)2 * n * 16 * 4) != cudaSuccess ||
      cudaMemset(x->epoch, 0, 16 * 4) != cudaSuccess || cudaMemset(x->err, 0, 16) != cudaSuccess) {
    set_error("peer exchange: cudaMemset failed");
    x->comm = nullptr;
    return fail(FLOCK_E_CUDA);
  }
  std::vector<float*> bufs(n, nullptr);
  std::vector<uint32_t*> flags(n, nullptr);
  bufs[rank] = x->buf;
  flags[rank] = x->flag;
  if (n > 1) {
    cudaIpcMemHandle_t mine[2];
    if (cudaIpcGetMemHandle(&mine[0], x->buf) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine[1], x->flag) != cudaSuccess) {
      set_error("peer exchange: cudaIpcGetMemHandle failed");
      x->comm = nullptr;
      return fail(FLOCK_E_CUDA);
    }
    std::vector<cudaIpcMemHandle_t> all((size_t)2 * n);
    int rc = flock_comm_allgather_bytes(c, mine, all.data(), (int64_t)sizeof(mine));
    if (rc) {
      x->comm = nullptr;
      return fail(rc);
    }
    int bad = -1;
    for (int r = 0; r < n && bad < 0; r++) {
      if (r == rank) continue;
      void* pb = nullptr;
      void* pf = nullptr;
      if (cudaIpcOpenMemHandle(&pb, all[(size_t)2 * r], cudaIpcMemLazyEnablePeerAccess) !=
          cudaSuccess) {
        bad = r;
        break;
      }
      x->opened.push_back(pb);
      if (cudaIpcOpenMemHandle(&pf, all[(size_t)2 * r + 1], cudaIpcMemLazyEnablePeerAccess) !=
          cudaSuccess) {
        bad = r;
        break;
      }
      x->opened.push_back(pf);
      bufs[r] = (float*)pb;
      flags[r] = (uint32_t*)pf;
    }
    cudaGetLastError();
    // every rank learns whether every rank mapped every peer
    float failed = bad >= 0 ? 1.0f : 0.0f, any = 0.0f;
    rc = flock_comm_allreduce_f32(c, &failed, &any, 1);
    if (rc || any > 0.0f) {
      if (bad >= 0) set_error("peer exchange: cannot map rank %d's memory (no peer access?)", bad);
      else if (!rc) set_error("peer exchange: another rank could not map its peers");
      x->comm = nullptr;  // the ranks agreed; no further collective here
      return fail(rc ? rc : FLOCK_E_UNSUPPORTED);
    }
  }
  if (cudaMemcpy(x->d_bufs, bufs.data(), (size_t)n * sizeof(float*), cudaMemcpyHostToDevice) !=
          cudaSuccess ||
      cudaMemcpy(x->d_flags, flags.data(), (size_t)n * sizeof(uint32_t*),
                 cudaMemcpyHostToDevice) != cudaSuccess) {
    set_error("peer exchange: pointer table upload failed");
    return fail(FLOCK_E_CUDA);  // every rank got here: the free's barrier is collective
  }
  *out = x;
  return FLOCK_OK;
}

int peer_xchg_run(PeerXchg* x, cudaStream_t st, float* h, const float* part, int64_t n) {
  if (x->failed) {
    set_error("tensor-parallel peer exchange failed earlier (a rank gave up waiting); free the "
              "model and set the exchange up again");
    return FLOCK_E_CUDA;
  }
  const int64_t ctas = (n + XCHG_CHUNK - 1) / XCHG_CHUNK;
  if (n > x->cap || n % 4 || ctas > XCHG_MAX_CTAS) {
    set_error("peer exchange of %lld floats: at most %lld (and %d per CTA x %d), a multiple of 4",
              (long long)n, (long long)x->cap, XCHG_CHUNK, XCHG_MAX_CTAS);
    return FLOCK_E_LIMIT;
  }
  k_peer_xchg<<<(unsigned)ctas, XCHG_THREADS, 0, st>>>(part, h, (int)n, x->rank, x->n, x->cap,
                                                       x->d_bufs, x->d_flags, x->epoch, x->err,
                                                       x->wait_ns);
  FLOCK_CK(cudaGetLastError());
  return FLOCK_OK;
}

// The device error word is sticky: once a wait ran out, this rank is an
// exchange behind (or ahead of) its peers, so every later check (and every
// later exchange) fails until the exchange is freed and set up again.
int peer_xchg_check(PeerXchg* x) {
  if (!x) return FLOCK_OK;
  if (!x->failed) {
    int e = 0;
    FLOCK_CK(cudaMemcpy(&e, x->err, 4, cudaMemcpyDeviceToHost));
    x->failed = e != 0;
  }
  if (x->failed) {
    set_error("tensor-parallel peer exchange gave up waiting for a rank; it stays failed until "
              "the model is freed and the exchange set up again");
    return FLOCK_E_CUDA;
  }
  return FLOCK_OK;
}

}  // namespace flock

using namespace flock;

extern "C" {

// One rank of an n_ranks exchange whose peers never publish (their buffers
// and flags are local allocations nothing writes): `calls` exchanges of n
// floats with a wait limit of wait_ms, each followed by the host check.
// Returns the last call's status (its message in flock_last_error): the
// first call gives up waiting, every later one is refused.  A test of the
// bounded wait and of the sticky failure that needs no second GPU.
int flock_op_peer_exchange_lone(flock_dev* d, int n_ranks, int64_t n, int wait_ms, int calls,
                                int* first_status) {
  if (!d || n_ranks < 2 || n_ranks > 8 || n < 4 || n % 4 || n > XCHG_CHUNK * XCHG_MAX_CTAS ||
      wait_ms < 1 || wait_ms > 2000 || calls < 1 || calls > 8)
    return FLOCK_E_ARG;
  FLOCK_CK(cudaSetDevice(d->ordinal));
  PeerXchg x;
  x.rank = 0;
  x.n = n_ranks;
  x.cap = n;
  x.wait_ns = (uint64_t)wait_ms * 1000000ull;
  DBuf bufs, flags, tab, epoch, err, part, h;
  const size_t buf_bytes = (size_t)2 * n_ranks * n * 4;
  const size_t flag_bytes = (size_t)2 * n_ranks * XCHG_MAX_CTAS * 4;
  FLOCK_TRY(bufs.alloc(buf_bytes * n_ranks));
  FLOCK_TRY(flags.alloc(flag_bytes * n_ranks));
  FLOCK_TRY(tab.alloc((size_t)2 * n_ranks * sizeof(void*)));
  FLOCK_TRY(epoch.alloc(16 * 4));
  FLOCK_TRY(err.alloc(16));
  FLOCK_TRY(part.alloc((size_t)n * 4));
  FLOCK_TRY(h.alloc((size_t)n * 4));
  FLOCK_CK(cudaMemset(flags.p, 0, flag_bytes * n_ranks));
  FLOCK_CK(cudaMemset(epoch.p, 0, 16 * 4));
  FLOCK_CK(cudaMemset(err.p, 0, 16));
  FLOCK_CK(cudaMemset(part.p, 0, (size_t)n * 4));
  FLOCK_CK(cudaMemset(h.p, 0, (size_t)n * 4));
  std::vector<void*> ptrs(2 * (size_t)n_ranks);
  for (int r = 0; r < n_ranks; r++) {
    ptrs[r] = bufs.as<uint8_t>() + (size_t)r * buf_bytes;
    ptrs[n_ranks + r] = flags.as<uint8_t>() + (size_t)r * flag_bytes;
  }
  FLOCK_CK(cudaMemcpy(tab.p, ptrs.data(), ptrs.size() * sizeof(void*), cudaMemcpyHostToDevice));
  x.d_bufs = tab.as<float*>();
  x.d_flags = reinterpret_cast<uint32_t**>(tab.as<void*>() + n_ranks);
  x.epoch = epoch.as<uint32_t>();
  x.err = err.as<int>();
  int rc = FLOCK_OK;
  for (int i = 0; i < calls; i++) {
    rc = peer_xchg_run(&x, d->stream, h.as<float>(), part.as<float>(), n);
    if (rc == FLOCK_OK) {
      FLOCK_CK(cudaStreamSynchronize(d->stream));
      rc = peer_xchg_check(&x);
    }
    if (i == 0 && first_status) *first_status = rc;
  }
  return rc;
}

}  // extern "C"

namespace flock {

}  // namespace flock
