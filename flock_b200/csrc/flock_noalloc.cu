// Greedy token selection that allocates nothing on the device.
//
// Who needs it: callers that hand this library device memory they already
// own and may not allocate more -- a host framework whose allocator owns the
// GPU's memory (a serving runtime that reserved it up front), a decode loop
// that must not call cudaMalloc between tokens because cudaMalloc
// synchronises the device and its latency is unbounded, or code that cannot
// reach the CUDA allocator at all (an FFI caller given raw device pointers).
// flock_op_argmax needs per-CTA scratch and takes it from its device handle,
// whose creation allocates; this entry point instead keeps that scratch in a
// fixed file-scope device array, sized for NOALLOC_MAX_CTAS partials.
//
// The array lives for as long as the library is loaded, on every GPU that
// loads it (8 KiB + 256 B).  All calls share it: two calls whose kernels
// overlap on the GPU race on the partials and the arrival counter, so the
// caller must order them (one stream, or events).  The counter is cleared
// before every launch; the partials are fully rewritten by each launch.
#include <cuda_runtime.h>

#include <mutex>

#include "flock_internal.h"
#include "ops.cuh"

namespace {

constexpr int NOALLOC_MAX_CTAS = 1024;      // partial (value, index) slots
constexpr int NOALLOC_PER_CTA = 4096;       // logits one CTA reduces at most
constexpr int64_t NOALLOC_MAX_N = (int64_t)NOALLOC_MAX_CTAS * NOALLOC_PER_CTA;

// [0, 4 KiB) partial values, [4 KiB, 8 KiB) partial indices, then the counter.
constexpr size_t OFF_VAL = 0, OFF_IDX = 4096, OFF_COUNT = 8192, SCRATCH_BYTES = 8192 + 256;
static __device__ __align__(256) unsigned char g_argmax_scratch[SCRATCH_BYTES];

// Device address of g_argmax_scratch per device ordinal, resolved once.
std::mutex g_mu;
void* g_addr[64] = {};

int scratch_address(int dev, void** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (dev < 0 || dev >= 64) {
    flock::set_error("device ordinal %d out of range", dev);
    return FLOCK_E_ARG;
  }
  if (!g_addr[dev]) {
    // The symbol's host-side name is not a device address: ask the runtime for
    // the address on the current device.
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_scratch);
    if (e != cudaSuccess || !p) {
      flock::set_error("cudaGetSymbolAddress(argmax scratch) failed: %s", cudaGetErrorString(e));
      return FLOCK_E_CUDA;
    }
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return FLOCK_OK;
}

}  // namespace

extern "C" {

int flock_argmax_noalloc(const float* x, int64_t n, int32_t* index_out, float* value_out,
                         void* stream) {
  if (!x || !index_out || !value_out || n < 1) {
    flock::set_error("argmax_noalloc: x, index_out and value_out must be device pointers, n >= 1");
    return FLOCK_E_ARG;
  }
  if (n > NOALLOC_MAX_N) {
    flock::set_error("argmax_noalloc: n = %lld exceeds the maximum %lld (%d scratch slots x %d "
                     "logits per slot); use flock_op_argmax", (long long)n,
                     (long long)NOALLOC_MAX_N, NOALLOC_MAX_CTAS, NOALLOC_PER_CTA);
    return FLOCK_E_LIMIT;
  }
  int dev = 0;
  FLOCK_CK(cudaGetDevice(&dev));
  void* base = nullptr;
  FLOCK_TRY(scratch_address(dev, &base));
  unsigned char* s = static_cast<unsigned char*>(base);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int sms = 148;
  FLOCK_CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  int64_t ctas = (n + 255) / 256;
  const int64_t need = (n + NOALLOC_PER_CTA - 1) / NOALLOC_PER_CTA;  // <= NOALLOC_MAX_CTAS
  if (ctas > 2 * sms) ctas = 2 * sms;
  if (ctas < need) ctas = need;
  if (ctas > NOALLOC_MAX_CTAS) ctas = NOALLOC_MAX_CTAS;
  FLOCK_CK(cudaMemsetAsync(s + OFF_COUNT, 0, sizeof(uint32_t), st));
  flock::k_argmax<<<(unsigned)ctas, 256, 0, st>>>(
      x, n, reinterpret_cast<float*>(s + OFF_VAL), reinterpret_cast<uint32_t*>(s + OFF_IDX),
      reinterpret_cast<uint32_t*>(s + OFF_COUNT), value_out, index_out, 0);
  FLOCK_CK(cudaGetLastError());
  return FLOCK_OK;
}

}  // extern "C"
