// Bulk-copy weight rings: each warp streams its share of a weight stream from HBM into
// its own ring of shared-memory stages with the TMA engine (cp.async.bulk, untiled,
// local memory only, no multicast) and waits on one mbarrier per stage.  Lane 0 issues
// a stage's copy; the whole warp consumes it from shared memory.
//
// Every wait is bounded: after QW_WAIT_LIMIT cycles the waiter records QW_DEVICE_TIMEOUT
// in the caller's status word and gives up, so a lost copy ends the kernel with an
// error the host can read instead of hanging the GPU.  A warp that gave up waits
// (bounded again) for its other copies in flight before it exits, so no copy can land
// in shared memory that a later CTA owns.
#pragma once

#include "qw_common.cuh"

namespace qw {

constexpr long long QW_WAIT_LIMIT = 1ll << 31;  // cycles (about a second at 2 GHz)
constexpr int QW_DEVICE_TIMEOUT = 1;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make barrier initialisation (generic proxy) visible to the TMA engine (async proxy).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// Order this thread's earlier generic accesses of shared memory before later
// async-proxy (bulk copy) writes to it.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// One arrival that also announces `bytes` of transaction count.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;\n"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Global -> shared bulk copy completing on `bar`; dst, src 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// try_wait suspends the thread (no issue slots used) until the phase completes or the
// hint (ns) passes; a waiting warp then does not take issue slots from computing warps.
constexpr uint32_t QW_SUSPEND_NS = 100000;

// The same copy with an L2 cache policy (e.g. evict-first for weights read once).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy) : "memory");
}

// L2 policy: lines of this access are evicted first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(QW_SUSPEND_NS)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of `bar`; false (and the status word set) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* status,
                                          long long limit = QW_WAIT_LIMIT) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) {
      if (status) atomicOr(status, QW_DEVICE_TIMEOUT);
      return false;
    }
  }
  return true;
}

// A warp's ring of NST stages of `stage_bytes` each in shared memory.
template <int NST>
struct WarpRing {
  uint8_t* buf;    // NST * stage_bytes
  uint64_t* bar;   // NST barriers (initialised with count 1)
  uint32_t stage_bytes;
  long long limit; // cycles a wait may take

  __device__ __forceinline__ uint8_t* stage(int q) const { return buf + (q % NST) * stage_bytes; }

  // Lane 0: start the copy of stage q (bytes <= stage_bytes) from src; weights read once
  // are copied with an evict-first L2 policy so they do not displace prefetched lines.
  __device__ __forceinline__ void issue(int q, const void* src, uint32_t bytes) const {
    uint64_t* b = bar + (q % NST);
    fence_proxy_async();
    mbar_arrive_expect_tx(b, bytes);
    bulk_g2s_hint(stage(q), src, bytes, b, l2_evict_first_policy());
  }
  // Lane 0: stage q from two sources, `bytes` each, into its two halves.
  __device__ __forceinline__ void issue2(int q, const void* src0, const void* src1, uint32_t bytes) const {
    uint64_t* b = bar + (q % NST);
    fence_proxy_async();
    mbar_arrive_expect_tx(b, 2 * bytes);
    const uint64_t pol = l2_evict_first_policy();
    bulk_g2s_hint(stage(q), src0, bytes, b, pol);
    bulk_g2s_hint(stage(q) + bytes, src1, bytes, b, pol);
  }
  // Whole warp: wait until stage q landed (bounded).
  __device__ __forceinline__ bool wait(int q, int32_t* status) const {
    return mbar_wait(bar + (q % NST), static_cast<uint32_t>((q / NST) & 1), status, limit);
  }
  // After a timeout: wait (bounded) for the stages [q0, q1) still in flight.
  __device__ __forceinline__ void drain(int q0, int q1) const {
    for (int q = q0; q < q1; ++q) {
      const long long t0 = clock64();
      while (!mbar_try_wait(bar + (q % NST), static_cast<uint32_t>((q / NST) & 1)))
        if (clock64() - t0 > limit) return;
    }
  }
};

}  // namespace qw
