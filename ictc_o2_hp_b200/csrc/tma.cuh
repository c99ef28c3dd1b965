// Bulk asynchronous copies (TMA, non-tensor form) and mbarrier helpers for sm_100a.
//
// Rows of the flat operands are contiguous, so a whole stage of rows moves with
// one `cp.async.bulk` per tensor (16-byte aligned addresses, sizes a multiple of
// 16 bytes).  No multicast is used anywhere.  Every wait is bounded in time:
// after kWaitLimitNs of the global nanosecond timer it records an error code in
// `g_ictc_device_error` and returns false, so a kernel can drain and exit instead
// of hanging.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ictc {

// Upper bound of one mbarrier wait: 2 s of %globaltimer.  A stage of a healthy
// kernel lands within microseconds, so only a copy that never completes reaches it.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
// Upper bound of each wait of the drain that follows a timed-out wait (copies
// already issued land before the CTA exits): 50 ms.
constexpr unsigned long long kDrainLimitNs = 50000000ull;

// Set to a nonzero code by a kernel whose bounded wait ran out.  Each translation
// unit that includes this header has its own copy; `take_unit_device_error` below
// reads and clears this unit's copy, each unit exports it under its own name and
// ictc_o2_device_error() consults every unit.
static __device__ int g_ictc_device_error;

// Host: reads and clears this translation unit's device error flag on the current
// device.  The caller synchronizes the device first.
[[maybe_unused]] static int take_unit_device_error(int* code, cudaError_t* err) {
  int value = 0;
  *err = cudaMemcpyFromSymbol(&value, g_ictc_device_error, sizeof(int));
  if (*err != cudaSuccess) return -1;
  const int zero = 0;
  *err = cudaMemcpyToSymbol(g_ictc_device_error, &zero, sizeof(int));
  if (*err != cudaSuccess) return -1;
  *code = value;
  return 0;
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
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

// Bounded wait for the phase with the given parity; false (and the device error
// flag set to `code`) when `limit_ns` of the global timer pass first.  The first
// poll is the common case and reads no timer.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_timer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
    }
    if (global_timer_ns() - start >= limit_ns) break;
  }
  atomicExch(&g_ictc_device_error, code);
  return false;
}

// Global -> shared bulk copy completing on `bar` (bytes counted by expect_tx).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace ictc
