// pipeline.cuh - mbarrier / bulk-copy primitives for sm_100a (inline PTX),
// with bounded waits.
//
// Every wait gives up after kWaitLimitNs of %globaltimer time (or at once when
// the CTA's abort word is set), ORs CNNUE_STATUS_TIMEOUT into the status word
// and returns false; callers keep their control flow (barrier counts stay
// matched) and only skip work, so a CTA always runs to its end.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace cnnue {
namespace pipe {

constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps until it completes or `hint_ns` passes, instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// mbar_wait whose retries sleep up to 20 us each (the wait limit still holds):
// for pipelines where many warps of an SM wait at once and spinning would
// take issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                uint32_t* status, unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (*abort) return false;
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (globaltimer() - t0 > limit_ns) {
      *abort = 1;
      atomicOr(status, CNNUE_STATUS_TIMEOUT);
      return false;
    }
  }
}

// Waits for the phase of `bar` with the given parity to complete.  Returns
// false (after flagging) on timeout or when *abort is set.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint32_t* status, unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (*abort) return false;
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > limit_ns) {
      *abort = 1;
      atomicOr(status, CNNUE_STATUS_TIMEOUT);
      return false;
    }
  }
}

// Teardown form of mbar_wait: ignores the abort word (it is used after an
// abort, to let copies or MMAs already in flight land before the CTA ends),
// still gives up after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, uint32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      atomicOr(status, CNNUE_STATUS_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Forms of the barrier and copy operations on raw shared-memory addresses
// (for loops that keep their addresses in registers).
__device__ __forceinline__ bool mbar_try_wait_addr(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_try_wait_sleep_addr(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}
// mbar_wait_sleep on a raw address.
__device__ __forceinline__ bool mbar_wait_addr(uint32_t bar, uint32_t parity, volatile int* abort, uint32_t* status,
                                               unsigned long long limit_ns) {
  if (mbar_try_wait_addr(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (*abort) return false;
    if (mbar_try_wait_sleep_addr(bar, parity, 20000u)) return true;
    if (globaltimer() - t0 > limit_ns) {
      *abort = 1;
      atomicOr(status, CNNUE_STATUS_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ void mbar_arrive_addr(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx_addr(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_copy_g2s_addr(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src),
      "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Orders this thread's earlier shared-memory accesses (and what it observed)
// before its later async-proxy operations on shared memory (bulk copies).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Publishes a monotonic counter after this warp's earlier shared-memory reads
// (call from one lane after __syncwarp()).
__device__ __forceinline__ void publish_counter(uint32_t* counter, uint32_t value) {
  __threadfence_block();
  *reinterpret_cast<volatile uint32_t*>(counter) = value;
}

// Waits until every counters[i] (i < n) is >= target.  Bounded like mbar_wait.
__device__ __forceinline__ bool wait_counters_reach(const uint32_t* counters, int n, uint32_t target,
                                                    volatile int* abort, uint32_t* status) {
  const volatile uint32_t* c = reinterpret_cast<const volatile uint32_t*>(counters);
  unsigned long long t0 = 0;
  for (uint32_t spin = 0;; ++spin) {
    bool ok = true;
    for (int i = 0; i < n; ++i) ok &= c[i] >= target;
    if (ok) {
      __threadfence_block();
      return true;
    }
    if (*abort) return false;
    if (spin == 0) t0 = globaltimer();
    if ((spin & 63) == 63) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        *abort = 1;
        atomicOr(status, CNNUE_STATUS_TIMEOUT);
        return false;
      }
      __nanosleep(64);
    }
  }
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` of
// transaction count on `bar` (no multicast).  dst/src 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace pipe
}  // namespace cnnue
