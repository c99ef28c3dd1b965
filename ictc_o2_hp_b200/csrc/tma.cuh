// Bulk asynchronous copies (TMA, non-tensor form) and mbarrier helpers for sm_100a.
//
// Rows of the flat operands are contiguous, so a whole stage of rows moves with
// one `cp.async.bulk` per tensor (16-byte aligned addresses, sizes a multiple of
// 16 bytes).  No multicast is used anywhere.  Every wait is bounded: after
// kSpinLimit polls it records an error code in `g_ictc_device_error` and returns
// false, so a kernel can drain and exit instead of hanging.
#pragma once

#include <cstdint>

namespace ictc {

constexpr long long kSpinLimit = 1ll << 28;  // polls; several seconds of waiting

// Set to a nonzero code by a kernel whose bounded wait ran out (one copy per
// translation unit; each unit exports a host reader, see common.cuh).
static __device__ int g_ictc_device_error;

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
// flag set to `code`) when the limit runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  for (long long i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
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
