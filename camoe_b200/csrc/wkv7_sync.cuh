// mbarrier, named-barrier and bulk-copy helpers with bounded waits.
//
// Every wait on an mbarrier gives up after kWaitLimitCycles (about a second
// at 1.9 GHz; g_wkv7_wait_limit), counts the event in g_wkv7_timeouts and
// reports failure, so a logic error can never leave a GPU spinning.  Callers stop their loops on a
// failed wait.  The counter is per translation unit (static); each kernel
// file exposes a host reader, summed by camoe_wkv7_device_errors().
#pragma once

#include <stdint.h>

namespace camoe {

static __device__ unsigned int g_wkv7_timeouts = 0;

constexpr long long kWaitLimitCycles = 2000000000LL;
// The limit in force (per translation unit, like the counter).  Only the
// test hook camoe_wkv7_test_hooks lowers it, to make a withheld arrival time
// out within milliseconds; it is read only once a wait has already failed its
// first try, so the fast path does not load it.
static __device__ long long g_wkv7_wait_limit = kWaitLimitCycles;

__device__ __forceinline__ uint32_t sm_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(sm_addr(bar)), "r"(count) : "memory");
}

// make barrier initialisation visible to the async proxy (bulk copies)
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n" ::"r"(sm_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;\n" ::"r"(sm_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(sm_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking test of the phase with the given parity: issued early, its
// result is read later, so the round trip overlaps other work.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(sm_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  const long long limit = *static_cast<volatile long long*>(&g_wkv7_wait_limit);
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > limit) {
      atomicAdd(&g_wkv7_timeouts, 1u);
      return false;
    }
  }
}

// 1-D bulk copy global -> shared of `bytes` (multiple of 16, both ends
// 16-byte aligned), completing on `bar` (complete_tx).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          sm_addr(dst)),
      "l"(src), "r"(bytes), "r"(sm_addr(bar))
      : "memory");
}

// Named barrier over `count` threads (a multiple of 32) of this CTA.
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also ANDs `pred` over the participating threads, so a
// group leaves a loop together when any member's wait has failed.
__device__ __forceinline__ bool named_sync_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

}  // namespace camoe

namespace camoe {

// 1-D bulk copy shared -> global (bulk-group completion), issued by one thread.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst),
               "r"(sm_addr(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
}
// wait until the issuing thread's bulk stores have finished reading shared memory
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
}
// wait until at most N of the issuing thread's most recent bulk-store groups
// are still reading shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read_n() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
// wait until the issuing thread's bulk stores have completed
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
}
// order this thread's generic-proxy shared-memory writes before later async-proxy reads
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

}  // namespace camoe
