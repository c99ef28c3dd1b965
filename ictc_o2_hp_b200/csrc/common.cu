// Status handling and device queries shared by all C-ABI launchers.
#include "common.cuh"

#include <mutex>

#include "tmap.cuh"

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

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode3(PFN_cuTensorMapEncodeTiled_v12000 fn, CUtensorMap* map, const float* base,
            uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0,
            uint32_t b1) {
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};  // bytes, dims 1 and 2
  const cuuint32_t box[3] = {b0, b1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1;
}

}  // namespace

int encode_row_tile_maps(const float* base, int64_t rows, int C, int M, bool full, bool cm,
                         int64_t width, int Ct, CUtensorMap* maps) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = tensor_map_encoder();
  if (fn == nullptr) return -1;
  const int s0 = full ? 2 : 1;
  const int copies = full ? 2 : 1;
  const uint64_t row_bytes = static_cast<uint64_t>(width) * 4;
  if (encode3(fn, &maps[0], base, C, s0, rows, static_cast<uint64_t>(C) * 4, row_bytes, Ct, s0))
    return -1;
  if (M == 0) {
    maps[1] = maps[0];
    return 0;
  }
  const float* fbase = base + static_cast<int64_t>(s0) * C;
  if (!cm)
    return encode3(fn, &maps[1], fbase, 2 * static_cast<uint64_t>(C), M * copies, rows,
                   static_cast<uint64_t>(C) * 8, row_bytes, 2 * Ct, M * copies);
  return encode3(fn, &maps[1], fbase, C, 2 * M * copies, rows, static_cast<uint64_t>(C) * 4,
                 row_bytes, Ct, 2 * M * copies);
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
