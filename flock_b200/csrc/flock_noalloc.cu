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
// fixed file-scope device array, sized for NOALLOC_MAX_CTAS partials.  The
// first call on a device loads the module (the runtime's lazy loading), so it
// must not be made while a stream is being captured.
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

// k_argmax walks its input with a grid stride, so the kernel itself handles
// any n whose indices fit its uint32 slots with up to NOALLOC_MAX_CTAS CTAs.
// NOALLOC_MAX_N is a bound this entry point chooses, not one the kernel
// needs: it covers every vocabulary (151,936 for Qwen3) with a wide margin
// and keeps the documented contract small.
constexpr int NOALLOC_MAX_CTAS = 1024;            // partial (value, index) slots
constexpr int64_t NOALLOC_MAX_N = 4194304;        // chosen bound (see above)

// [0, 4 KiB) partial values, [4 KiB, 8 KiB) partial indices, then the counter.
constexpr size_t OFF_VAL = 0, OFF_IDX = 4096, OFF_COUNT = 8192, SCRATCH_BYTES = 8192 + 256;
static __device__ __align__(256) unsigned char g_argmax_scratch[SCRATCH_BYTES];

// SM count per device ordinal (a property of the GPU, not of its context).
std::mutex g_mu;
int g_sms[64] = {};

int sm_count(int dev, int* out) {
  if (dev < 0 || dev >= 64) {
    flock::set_error("device ordinal %d out of range", dev);
    return FLOCK_E_ARG;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_sms[dev]) {
    int n = 0;
    FLOCK_CK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    g_sms[dev] = n > 0 ? n : 1;
  }
  *out = g_sms[dev];
  return FLOCK_OK;
}

// The scratch array's device address in the current context, asked for on
// every call: an address cached across calls would go stale if the primary
// context were torn down and made again (cudaDeviceReset).  Once the module
// is loaded the query is a table lookup in the runtime.
int scratch_address(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_scratch);
  if (e != cudaSuccess || !p) {
    flock::set_error("cudaGetSymbolAddress(argmax scratch) failed: %s", cudaGetErrorString(e));
    return FLOCK_E_CUDA;
  }
  *out = p;
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
    flock::set_error("argmax_noalloc: n = %lld exceeds the maximum %lld this entry point "
                     "accepts; use flock_op_argmax", (long long)n, (long long)NOALLOC_MAX_N);
    return FLOCK_E_LIMIT;
  }
  int dev = 0;
  FLOCK_CK(cudaGetDevice(&dev));
  void* base = nullptr;
  FLOCK_TRY(scratch_address(&base));
  unsigned char* s = static_cast<unsigned char*>(base);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int sms = 0;
  FLOCK_TRY(sm_count(dev, &sms));
  // two CTAs per SM at most (the grid stride covers the rest), one per 256
  // logits for small inputs
  int64_t ctas = (n + 255) / 256;
  if (ctas > 2 * (int64_t)sms) ctas = 2 * (int64_t)sms;
  if (ctas > NOALLOC_MAX_CTAS) ctas = NOALLOC_MAX_CTAS;
  FLOCK_CK(cudaMemsetAsync(s + OFF_COUNT, 0, sizeof(uint32_t), st));
  flock::k_argmax<<<(unsigned)ctas, 256, 0, st>>>(
      x, n, reinterpret_cast<float*>(s + OFF_VAL), reinterpret_cast<uint32_t*>(s + OFF_IDX),
      reinterpret_cast<uint32_t*>(s + OFF_COUNT), value_out, index_out, 0);
  FLOCK_CK(cudaGetLastError());
  return FLOCK_OK;
}

}  // extern "C"
