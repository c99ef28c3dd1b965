// Test hook for the bounded mbarrier wait every staged kernel uses: one CTA of one
// warp initialises an mbarrier that nothing ever arrives at, waits on it with the
// same helper the kernels use (tma.cuh) under a caller-given limit, and when the
// limit runs out records its code in the device error flag and returns.  No copy
// is issued, so nothing is in flight when the CTA exits.  This shows, on the GPU,
// that a wait which can never complete ends with a status the host reads instead
// of hanging.
#include "common.cuh"
#include "tma.cuh"

namespace ictc {

namespace {

constexpr int kProbeCode = 13;

__global__ void wait_probe_kernel(unsigned long long limit_ns, int* waited_ok) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) *waited_ok = mbar_wait(&bar, 0, kProbeCode, limit_ns) ? 1 : 0;
}

}  // namespace

int probe_take_device_error(int* code) {
  cudaError_t e;
  if (take_unit_device_error(code, &e) != 0) return cuda_fail(e, "probe device error flag");
  return ICTC_OK;
}

}  // namespace ictc

using namespace ictc;

extern "C" int32_t ictc_o2_test_wait_timeout(int32_t limit_us, int32_t* waited_ok,
                                             void* stream) {
  if (limit_us < 1 || limit_us > 1000000)
    return fail(ICTC_ERR_INVALID, "limit_us must be in [1, 1000000], got %d", limit_us);
  if (waited_ok == nullptr || !aligned(waited_ok, 4))
    return fail(ICTC_ERR_INVALID, "waited_ok must be a 4-byte aligned device pointer");
  wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(limit_us) * 1000ull, waited_ok);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "wait probe launch");
}
