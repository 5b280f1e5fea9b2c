// Asynchronous bulk-copy (TMA, non-tensor form) and mbarrier helpers for sm_100a.
//
// cp.async.bulk moves a contiguous, 16-byte aligned range of global memory into shared memory
// and signals an mbarrier with the number of bytes delivered, so one issuing thread keeps tens of
// kilobytes per SM in flight while the other warps compute.  Every wait here is bounded: after
// kWaitLimitNs of global time it records a fault in g_b200_fault and returns false, so a kernel
// never spins forever (the caller keeps going with whatever data it has, finishes its normal
// control flow, and the host reads the fault with b200_device_fault()).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

// Fault word shared by every kernel of the library: bit k set = fault kind k seen.
__device__ unsigned int g_b200_fault;

enum FaultBits : unsigned {
  kFaultWaitTimeout = 1u,   // a bounded mbarrier / flag wait gave up
  kFaultNoTensorCore = 2u,  // a tensor-core kernel ran from code built without sm_100a features
};

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async proxy (bulk copies, tensor cores).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread may sleep (up to `hint_ns`) until the phase
// completes instead of returning at once, so a waiting warp takes no issue slots from the warps
// that have work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait that sleeps between polls (see mbar_try_wait_sleep); for warps whose wait overlaps
// other warps' work.  Returns false (and records kFaultWaitTimeout) after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity) {
  constexpr uint32_t kHintNs = 1000000u;  // 1 ms; the hardware wakes the thread when the phase completes
  if (mbar_try_wait_sleep(bar, parity, kHintNs)) return true;
  const unsigned long long t0 = global_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, kHintNs)) return true;
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_b200_fault, kFaultWaitTimeout);
      return false;
    }
  }
}

// Wait until the barrier phase with the given parity has completed.  Returns false (and records
// kFaultWaitTimeout) after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_b200_fault, kFaultWaitTimeout);
      return false;
    }
  }
}

// Global -> shared bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned); the
// bytes are counted against `bar`'s transaction count.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Shared -> global bulk copy (both addresses 16-byte aligned, bytes a multiple of 16), tracked by
// the issuing thread's bulk-async groups.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_addr(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's committed bulk groups still read their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until all of this thread's committed bulk groups have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Orders this thread's earlier generic-proxy shared-memory accesses before later async-proxy
// (bulk copy / TMA) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier over `count` threads (a subset of the CTA).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace b200
