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

int allow_smem(const void* kernel, size_t bytes) {
  static std::mutex mu;
  static const void* seen[256] = {};
  static size_t granted[256] = {};
  std::lock_guard<std::mutex> lock(mu);
  int slot = -1;
  for (int i = 0; i < 256; ++i) {
    if (seen[i] == kernel) {
      if (granted[i] >= bytes) return ICTC_OK;
      slot = i;
      break;
    }
    if (seen[i] == nullptr) {
      slot = i;
      break;
    }
  }
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  if (slot >= 0) {
    seen[slot] = kernel;
    granted[slot] = bytes;
  }
  return ICTC_OK;
}

}  // namespace ictc

extern "C" const char* ictc_o2_last_error(void) { return ictc::g_message; }

extern "C" int32_t ictc_o2_device_error(int32_t* code) {
  if (code == nullptr) return ictc::fail(ICTC_ERR_INVALID, "code is null");
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return ictc::cuda_fail(e, "cudaDeviceSynchronize");
  // every unit's flag is read and cleared; the first nonzero code is reported
  int (*const units[])(int*) = {ictc::tp_take_device_error, ictc::uvu_take_device_error,
                                ictc::radial_take_device_error, ictc::probe_take_device_error};
  int first = 0;
  for (auto take : units) {
    int value = 0;
    const int st = take(&value);
    if (st != ICTC_OK) return st;
    if (first == 0) first = value;
  }
  *code = first;
  return ICTC_OK;
}

extern "C" int32_t ictc_o2_abi_version(void) { return 102; }
