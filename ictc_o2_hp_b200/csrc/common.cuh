// Shared helpers for the C-ABI launchers: status codes, the per-thread error
// message, device properties and small device utilities.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "ictc_o2_b200.h"

namespace ictc {

// Records a formatted message for ictc_o2_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Converts a CUDA error (launch or query) into ICTC_ERR_CUDA with its name.
int cuda_fail(cudaError_t err, const char* what);

// SM count and the current device; cached per device.
int sm_count(int device);

// Each translation unit whose kernels hold bounded waits reads and clears its own
// copy of the device error flag on the current device (nonzero: a bounded wait ran
// out); the caller synchronizes the device first.
int tp_take_device_error(int* code);
int uvu_take_device_error(int* code);
int radial_take_device_error(int* code);
int probe_take_device_error(int* code);

// Opts a kernel into `bytes` of dynamic shared memory (cached per kernel).
int allow_smem(const void* kernel, size_t bytes);

inline bool aligned(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Row layout of a flat TensorProduct operand ([N, width], layout 0 of the
// reference, triton_o2.py:110-112): [0e: C][0o: C, full only][m = 1..M:
// copies x C x 2].
struct TpLayout {
  int C;
  int64_t width;
  int fbase;    // offset of frequency 1
  int fstride;  // offset step between consecutive frequencies
  int cm;       // frequency blocks stored [copy][component][channel] (1) or
                // [copy][channel][component] (0)
};

inline TpLayout tp_layout(int C, int m_max, bool full, int cm = 0) {
  TpLayout L;
  L.C = C;
  L.cm = cm;
  L.fbase = full ? 2 * C : C;
  L.fstride = full ? 4 * C : 2 * C;
  L.width = static_cast<int64_t>(L.fbase) + static_cast<int64_t>(m_max) * L.fstride;
  return L;
}

// Normalization-dependent magnitude of each path class (see o2_paths.cuh).
struct Mags {
  float m[4];
};

inline Mags tp_mags(int normalization) {
  const float r = 0.70710678118654752440f;
  Mags g;
  if (normalization == ICTC_NORM_COMPONENT) {
    g.m[0] = 1.0f; g.m[1] = 1.0f; g.m[2] = r; g.m[3] = r;
  } else {
    g.m[0] = 1.0f; g.m[1] = r; g.m[2] = r; g.m[3] = 0.5f;
  }
  return g;
}

// Prefetch of the 128-byte line holding p into L1 (a hint; p must be a valid
// address of the tensor it points into).
__device__ __forceinline__ void prefetch_l1(const float* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// Paired FP32 multiply-add: c + a * b componentwise as one sm_100 f32x2 FMA.
// Each component is rounded exactly as fmaf(a, b.x, c.x) / fmaf(a, b.y, c.y), so
// paired and scalar code give bit-identical results; the pair takes one issue
// slot instead of two.  The outer-product (GEMM) cores keep their accumulators as
// float2 pairs along the column index and use this for every k step.
__device__ __forceinline__ float2 fma2(float a, float2 b, float2 c) {
  return __ffma2_rn(make_float2(a, a), b, c);
}

// Element j of a row of paired accumulators (j a compile-time constant after
// unrolling, so this is a register name, not a select).
template <int N>
__device__ __forceinline__ float pair_at(const float2 (&v)[N], int j) {
  return (j & 1) ? v[j >> 1].y : v[j >> 1].x;
}

}  // namespace ictc
