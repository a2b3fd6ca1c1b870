// mbarrier, bulk-copy and timer primitives shared by the persistent decode
// kernel and the tensor-core GEMM.  Every wait is bounded in global time so
// a kernel that loses a producer returns with an error flag instead of
// hanging the GPU.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace flock {

constexpr uint64_t WAIT_NS = 2000000000ull;    // a wait gives up after 2 s
constexpr uint32_t WAIT_MAX_POLLS = 1u << 26;  // backstop on the poll count

FLOCK_DEV uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
FLOCK_DEV void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
FLOCK_DEV void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes) : "memory");
}
// Adds `bytes` to the transaction count without arriving.
FLOCK_DEV void mbar_expect_tx_only(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes) : "memory");
}
FLOCK_DEV void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
FLOCK_DEV bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
FLOCK_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// try_wait that lets the hardware suspend the thread for up to `hint_ns`
// while the phase is incomplete (it resumes as soon as the phase completes),
// so a waiting warp stops taking issue slots from the warps that compute.
FLOCK_DEV bool mbar_try_wait_sleep(uint64_t* b, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: false after WAIT_NS of global time (or WAIT_MAX_POLLS polls),
// or as soon as *err is set when `watch_err`.  The first WAIT_SPIN polls
// return at once (short waits stay short); later polls may sleep up to
// WAIT_SLEEP_NS so a long-waiting warp yields its issue slots.
constexpr uint32_t WAIT_SLEEP_NS = 20000;
constexpr uint32_t WAIT_SPIN = 4096;
FLOCK_DEV bool mbar_wait(uint64_t* b, uint32_t parity, const int* err, bool watch_err = true) {
  uint64_t t0 = 0;
  for (uint32_t i = 0; i < WAIT_MAX_POLLS; i++) {
    if (i < WAIT_SPIN ? mbar_try_wait(b, parity) : mbar_try_wait_sleep(b, parity, WAIT_SLEEP_NS))
      return true;
    if ((i & 63) == 63) {
      if (watch_err && *(volatile const int*)err) return false;
      const uint64_t now = globaltimer_ns();
      if (!t0) t0 = now;
      else if (now - t0 > WAIT_NS) return false;
    }
  }
  return false;
}
// Bounded wait that never asks the hardware to suspend the thread for long:
// for latency-critical pipelines where a late wake-up costs more than the
// issue slots of polling (a producer that must refill a ring slot as soon as
// it drains, consumers that must start on a slot as soon as it fills).
FLOCK_DEV bool mbar_wait_poll(uint64_t* b, uint32_t parity, const int* err, bool watch_err = true) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; i++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 63) == 63) {
      if (watch_err && *(volatile const int*)err) return false;
      const uint64_t now = globaltimer_ns();
      if (!t0) t0 = now;
      else if (now - t0 > WAIT_NS) return false;
    }
  }
}
// Orders this thread's generic shared-memory writes before later async-proxy
// reads of them (bulk copies, tensor-core operand reads).
FLOCK_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
FLOCK_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
}  // namespace flock
