// Bulk-copy pipeline primitives for sm_100a: mbarrier ring + cp.async.bulk
// (TMA bulk copies global -> shared, no multicast).
//
// Every wait is bounded: after kWaitLimitNs of %globaltimer time a waiter
// gives up, records an LG_ERR_TIMEOUT status word with the stage that gave
// up, and returns false so the kernel can leave instead of hanging.
#pragma once
#include "common.cuh"

namespace lg {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// status word codes: LG_ERR_TIMEOUT (6) in the low byte, the waiting site above it
enum WaitSite : int {
  kSiteGuFull = 1 << 8, kSiteGuEmpty = 2 << 8, kSiteGuDrain = 3 << 8,
  kSiteDnFull = 4 << 8, kSiteDnEmpty = 5 << 8, kSiteDnDrain = 6 << 8,
  kSiteSelfTestBar = 30 << 8, kSiteSelfTestFlag = 31 << 8,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity, int* status, int site,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(b, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(b, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) {
      if (status) atomicExch(status, 6 | site);
      return false;
    }
  }
  return true;
}
// Bounded wait until the global word *flag is nonzero (acquire loads, polls
// backed off by poll_ns); on timeout the status word records 6 | site.
__device__ __forceinline__ bool flag_wait(const unsigned* flag, int* status, int site,
                                          unsigned long long limit_ns = kWaitLimitNs, unsigned poll_ns = 256) {
  auto load = [&] {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    return v;
  };
  if (load()) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!load()) {
    if (globaltimer_ns() - t0 > limit_ns) {
      if (status) atomicExch(status, 6 | site);
      return false;
    }
    __nanosleep(poll_ns);
  }
  return true;
}
// mbar_wait by every lane of a warp with a warp-uniform result, so the
// shuffles that follow never see lanes that disagree about a timeout
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* b, unsigned parity, int* status, int site,
                                               unsigned long long limit_ns = kWaitLimitNs) {
  return __all_sync(0xffffffffu, mbar_wait(b, parity, status, site, limit_ns));
}
// contiguous global -> shared copy completing `bytes` of transactions on `bar`;
// dst, src and bytes must be multiples of 16
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Named barrier `id` over `nthreads` threads that also ANDs a flag over them:
// every participant gets the same verdict, so a group of warps leaves a loop
// together (a warp that left alone would strand the others at the group's
// next named barrier).
__device__ __forceinline__ bool named_and(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}
// named barrier `id` (1..15) over `nthreads` threads of the CTA.  The
// non-.aligned form: threads arrive one by one, so it is correct right after
// code where one lane of a warp took a different path (bar.sync, the .aligned
// form, requires a converged warp).
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace lg
