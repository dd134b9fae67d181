// Bulk-copy (TMA, non-tensor) and mbarrier primitives for sm_100a, written
// as inline PTX, plus the bounded wait every pipelined kernel uses.
//
// A kernel stages its input rows global -> shared with
// cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes: one
// instruction moves a whole contiguous block (a token's head rows, a hidden
// row), the copy engine does the addressing, and completion is counted in
// bytes on an mbarrier in shared memory. No multicast form is used anywhere.
//
// Rules these helpers rely on (PTX ISA, bulk copies): source and destination
// 16-byte aligned, size a multiple of 16; shared memory that generic loads
// have read must be fenced (fence.proxy.async) before the async proxy writes
// it again; an initialised mbarrier is published with
// fence.mbarrier_init before the copy engine signals it.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace bloth {

// Bit set in the device fault word when a kernel gave up waiting for a bulk
// copy (bloth_device_fault() reads it).
constexpr unsigned kFaultCopyTimeout = 1u;
// Bit set when, after such an expired wait, a kernel also gave up waiting for
// the copies it had already issued (so a copy may have still been in flight
// when it returned).
constexpr unsigned kFaultDrainTimeout = 2u;
// A bulk-copy completion wait gives up after this long (the copies it waits
// for complete in microseconds; this only bounds a broken launch).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arrive (count 1) and add `bytes` to the transaction count of the current phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Test-and-wait on phase `parity`: the thread is suspended (issuing nothing)
// until the phase completes or about `kSuspendNs` pass, whichever is first,
// so warps waiting for their copies leave the issue slots to warps that
// compute.
constexpr uint32_t kSuspendNs = 1000000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for phase `parity` of `bar` to complete. Returns false (and records
// kFaultCopyTimeout in *fault, the library's device fault word) if it has not
// completed within limit_ns (kWaitLimitNs unless a caller asks for less).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* fault,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > limit_ns) {
      if (fault != nullptr) atomicOr(fault, kFaultCopyTimeout);
      return false;
    }
  }
  return true;
}

// After a wait on ring slot `sl` (phase `ph`) gave up: waits, each with the
// same bound, for the `inflight` slots issued from `sl` on (sl included, the
// ring wrapping after `nst` slots and flipping the phase), so that no bulk
// copy this thread's CTA issued is still writing its shared memory when the
// kernel returns. A wait that gives up here too records kFaultDrainTimeout.
__device__ __forceinline__ void drain_ring(uint64_t* bars, int nst, int sl, uint32_t ph,
                                           int inflight, unsigned int* fault,
                                           unsigned long long limit_ns = kWaitLimitNs) {
  for (int k = 0; k < inflight; ++k) {
    if (!mbar_wait(&bars[sl], ph, nullptr, limit_ns) && fault != nullptr)
      atomicOr(fault, kFaultDrainTimeout);
    if (++sl == nst) {
      sl = 0;
      ph ^= 1u;
    }
  }
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned) that signals `bar` on completion.
__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// L2 policy that marks lines as first to evict: for inputs a kernel reads
// exactly once, so that they do not displace lines still in use.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// bulk_load with an L2 cache policy (from evict_first_policy()).
__device__ __forceinline__ void bulk_load_hint(void* dst_smem, const void* src, uint32_t bytes,
                                               uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1], %2, [%3], %4;" ::"r"(smem_addr(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <typename T, int VEC>
__device__ __forceinline__ Pack<T, VEC> lds_pack(const unsigned char* p) {
  return *reinterpret_cast<const Pack<T, VEC>*>(p);
}

}  // namespace bloth
