// Bulk-copy (TMA engine, 1-D cp.async.bulk) and mbarrier helpers for sm_100a.
// Every wait is bounded by the global timer: on timeout it records `code` in
// the device error word and returns false, so a kernel never spins forever.
#pragma once
#include <cstdint>

namespace fg {

// Error codes written to the device error word.
enum DevErr { DEVERR_NONE = 0, DEVERR_GEMV_FULL = 1, DEVERR_GEMV_EMPTY = 2, DEVERR_ATTN_FULL = 3,
              DEVERR_ATTN_EMPTY = 4, DEVERR_DRAIN = 5, DEVERR_GRID = 6 };
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Make barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait with a suspend-time hint: a waiting warp sleeps in hardware until
// the phase completes (or ~0.5 ms pass) instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(500000u)
      : "memory");
  return ok != 0;
}
// Wait for the phase of `parity` to complete; false (and err = code) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 4; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (err && *(volatile int *)err != 0) return false;  // another CTA already failed: stop early
    if (global_ns() - t0 > kWaitTimeoutNs) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// try_wait that suspends for at most ~100 ns: for a single thread whose wake-up
// latency is on the critical path (the hardware may resume a long-suspended
// thread hundreds of cycles after the phase completes).
__device__ __forceinline__ bool mbar_try_wait_short(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(100u)
      : "memory");
  return ok != 0;
}
// mbar_wait with short suspends; the same bounds.
__device__ __forceinline__ bool mbar_wait_poll(uint64_t *bar, uint32_t parity, int *err, int code) {
  if (mbar_try_wait_short(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait_short(bar, parity)) return true;
    if (err && *(volatile int *)err != 0) return false;  // another CTA already failed: stop early
    if (global_ns() - t0 > kWaitTimeoutNs) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// Wait for a phase during a drain: bounded by time only (a drain must wait
// for copies in flight even after another thread reported an error).
__device__ __forceinline__ void mbar_wait_drain(uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitTimeoutNs) return;
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Global -> shared bulk copy; `bytes` and both addresses multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Barrier among the first `threads` threads of the CTA (named barrier 1).
__device__ __forceinline__ void named_sync(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}
// Named barrier `id` (1..15) over `threads` threads (a multiple of 32).
__device__ __forceinline__ void named_sync_id(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace fg
