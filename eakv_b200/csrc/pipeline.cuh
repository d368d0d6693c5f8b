// pipeline.cuh - mbarrier + bulk-copy (TMA, cp.async.bulk) primitives used by
// the decode kernels, written as inline PTX for sm_100a.
//
// Every wait is bounded: a wait that runs out of its iteration budget
// returns false, the caller records it in the device status word and
// leaves, so a broken pipeline can never hang the GPU.
#pragma once
#include <stdint.h>

namespace eakv {

constexpr uint32_t kWaitBudget = 1u << 22;   // try_wait polls before giving up
constexpr int kStatusWaitTimeout = 1;
constexpr int kStatusBadIndex = 2;
constexpr int kStatusLateCopy = 4;   // a stage still had a copy in flight at the end

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete: at most
// `budget` polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t budget) {
  for (uint32_t i = 0; i < budget; i++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Bounded wait that suspends instead of spinning: each try may sleep up to
// about 2 us and returns as soon as the phase completes; at most `budget`
// tries. For waits that are expected to take a while (a warp waiting on
// tensor-core work or on other warps), so that the waiting warp does not
// take issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_wait_sleep(uint32_t bar, uint32_t parity, uint32_t budget) {
  for (uint32_t i = 0; i < budget; i++) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(2000u)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// Bounded wait until page i has been requested into its stage (last = the
// stage's "last page requested" slot). Only then is the stage's barrier in
// page i's phase: a consumer that waited on the phase parity earlier, while
// the barrier was still in the phase of the page two uses back, would see
// that older phase (same parity) as complete. Pages enter a stage in
// increasing order and page i + nstage only after page i was consumed, so
// the slot never passes i before this wait.
__device__ __forceinline__ bool wait_requested(const int *last, int i, uint32_t budget) {
  const volatile int *p = last;
  for (uint32_t k = 0; k < budget; k++)
    if (*p >= i) {
      __threadfence_block();
      return true;
    }
  return false;
}

// Publishes "page i requested into this stage" after the barrier arrive and
// the copies were issued (read by wait_requested).
__device__ __forceinline__ void publish_requested(int *last, int i) {
  __threadfence_block();
  *reinterpret_cast<volatile int *>(last) = i;
}

// True when no stage has a copy in flight: the phase of the last page
// requested into every stage has completed (one non-blocking test each).
__device__ __forceinline__ bool stages_idle(const uint64_t *bars, const int *last, int nstage) {
  bool idle = true;
  for (int s = 0; s < nstage; s++)
    if (last[s] >= 0 && !mbar_try_wait(smem_u32(&bars[s]), (last[s] / nstage) & 1)) idle = false;
  return idle;
}

// After a wait ran out: wait (bounded again) for the last copy requested
// into every stage, so that no bulk copy still writes this CTA's shared
// memory when it exits. last[s] is the page last requested into stage s
// (-1: none); its phase parity is (last[s] / nstage) & 1, and a phase that
// completed earlier answers at once.
__device__ __forceinline__ void drain_stages(const uint64_t *bars, const int *last, int nstage,
                                             uint32_t budget) {
  for (int s = 0; s < nstage; s++)
    if (last[s] >= 0) mbar_wait(smem_u32(&bars[s]), (last[s] / nstage) & 1, budget);
}

// 1-D bulk copy global -> shared, completion counted in bytes on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// its later async-proxy (bulk copy) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Stage release without waiting: every consumer warp calls this (lane 0)
// after its last read of a stage; the call that completes the set returns
// true exactly once, resets the counter, and its caller refills the stage.
// Every value a warp loaded from the stage has been consumed by the time it
// releases it, so those reads are complete; the counter itself is updated
// atomically. The proxy fence orders them before the refill's async write.
__device__ __forceinline__ bool stage_release_last(int *counter, int n_warps) {
  const int old = atomicAdd(counter, 1);
  if (old != n_warps - 1) return false;
  *counter = 0;
  fence_proxy_async_smem();
  return true;
}

// Named barrier over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace eakv
