// Status handling and device queries shared by all C-ABI launchers.
#include "common.cuh"

#include <mutex>

namespace ictc {

namespace {
thread_local char g_message[1024] = "no error";
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(ICTC_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}

int sm_count(int device) {
  static std::mutex mu;
  static int cache[64] = {};
  if (device < 0 || device >= 64) return 1;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n < 1)
      n = 1;
    cache[device] = n;
  }
  return cache[device];
}

}  // namespace ictc

extern "C" const char* ictc_o2_last_error(void) { return ictc::g_message; }

extern "C" int32_t ictc_o2_abi_version(void) { return 100; }
