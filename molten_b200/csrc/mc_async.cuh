// Asynchronous-copy and synchronisation primitives (inline PTX, sm_90+/sm_100a):
// mbarriers, 1-D bulk copies global -> shared (cp.async.bulk, the TMA engine's
// untiled form), and bounded device-scope flag waits.
//
// Every wait here is bounded: after `limit` polls it gives up and returns
// false, and callers record an error status instead of hanging the GPU.
#pragma once
#include <stdint.h>

__device__ __forceinline__ uint32_t mc_smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mc_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(mc_smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (the bulk copies).
__device__ __forceinline__ void mc_fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mc_mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mc_smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mc_mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(mc_smem_u32(bar)) : "memory");
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void mc_bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(mc_smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(mc_smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 policy that leaves the default eviction priority.
__device__ __forceinline__ uint64_t mc_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_unchanged.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// L2 policy for data read exactly once (streamed weights).
__device__ __forceinline__ uint64_t mc_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ bool mc_mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(mc_smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Like mc_mbar_test, but the thread may be suspended (up to `hint_ns`) until
// the phase completes, so waiting warps do not take issue slots from the
// warps doing work.
__device__ __forceinline__ bool mc_mbar_test_sleep(uint64_t* bar, uint32_t parity,
                                                   uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(mc_smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` to complete; false after `limit` polls.
__device__ __forceinline__ bool mc_mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit) {
  for (uint32_t it = 0; it < limit; ++it) {
    if (mc_mbar_test(bar, parity)) return true;
  }
  return false;
}

__device__ __forceinline__ uint32_t mc_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void mc_red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Spins (one thread) until *p >= target; false after `limit` polls.
__device__ __forceinline__ bool mc_wait_geq(const uint32_t* p, uint32_t target, uint32_t limit) {
  for (uint32_t it = 0; it < limit; ++it) {
    if (mc_ld_acquire(p) >= target) return true;
    __nanosleep(32);
  }
  return false;
}

// 16-byte asynchronous copy global -> shared (LDGSTS), L2-only caching.
__device__ __forceinline__ void mc_cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(mc_smem_u32(dst)), "l"(src)
               : "memory");
}

// Arrives on `bar` once all of this thread's prior cp.async copies landed
// (the arrival counts against the barrier's expected count).
__device__ __forceinline__ void mc_cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(mc_smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mc_cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Polling loads of words another CTA publishes: asm volatile so the load is
// issued on every poll (a non-volatile load may be hoisted out of the loop),
// and the matching L2 stores.
__device__ __forceinline__ unsigned long long mc_ld_poll_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Two 64-bit words in one 16-byte load; each word is read whole (a tagged
// value published by one 64-bit store is never torn).
__device__ __forceinline__ void mc_ld_poll_v2u64(const unsigned long long* p,
                                                 unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ uint4 mc_ld_poll_v4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ void mc_st_publish_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.global.cg.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void mc_st_publish_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.global.cg.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
