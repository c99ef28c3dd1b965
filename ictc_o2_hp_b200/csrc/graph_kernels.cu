// Message-passing plumbing around the radial product: row gathers and
// deterministic segment sums.
//
// A message-passing layer gathers node features by each edge's source
// (x_e = nodes[src_e]), runs the edge product, and sums the messages into the
// destination nodes (out_n = sum over edges with dst_e = n).  The reference keeps
// both steps outside its chain (docs/RADIAL.md:97-99); here they are kernels with
// fixed summation order, so that a layer's outputs and node gradients are
// bit-identical from run to run:
//   gather_rows:  out[r, :] = source[index[r], :]
//   segment_sum:  out[s, :] = sum over e in [offsets[s], offsets[s+1]) of
//                 values[order ? order[e] : e, :], added in increasing e
// The segment sum is also the adjoint of the gather (node gradients = segment sum
// of edge gradients grouped by source) and the gather the adjoint of the segment
// sum, so one pair of kernels serves both directions.
//
// Both kernels are HBM-bound streams: one warp per output row, 16-byte column
// chunks when the width and pointers allow (the segment sum then keeps each lane's
// columns in registers across the segment's edges), plain loads otherwise.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace ictc {
namespace {

constexpr int kGraphThreads = 256;

__global__ void __launch_bounds__(kGraphThreads) gather_rows_kernel(
    const float* __restrict__ source, const int64_t* __restrict__ index, float* __restrict__ out,
    int64_t rows, int64_t width, int64_t source_rows, bool vec, int* bad) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kGraphThreads / 32);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (kGraphThreads / 32) + (threadIdx.x >> 5);
       r < rows; r += warps) {
    const int64_t src = __ldg(index + r);
    float* dst = out + r * width;
    if (src < 0 || src >= source_rows) {  // out of range: zeros, and report it
      if (lane == 0) atomicExch(bad, 1);
      for (int64_t c = lane; c < width; c += 32) dst[c] = 0.f;
      continue;
    }
    const float* row = source + src * width;
    if (vec) {
      const float4* s4 = reinterpret_cast<const float4*>(row);
      float4* d4 = reinterpret_cast<float4*>(dst);
      for (int64_t c = lane; c < width / 4; c += 32) d4[c] = __ldg(s4 + c);
    } else {
      for (int64_t c = lane; c < width; c += 32) dst[c] = __ldg(row + c);
    }
  }
}

// 16-byte segment sum with each lane's column block in registers: a warp reads up to 32
// edge indices of its segment at once (one per lane) and hands them out by shuffle, then
// every lane loads its K float4 columns of one edge row together, so K loads per lane
// are in flight per edge instead of one index load and one value load in sequence.
// Columns are summed over the segment's edges in increasing e, as segment_sum_kernel
// does: the results are bit-identical.
constexpr int kSegCols = 8;  // float4 columns per lane held in registers

__global__ void __launch_bounds__(kGraphThreads) segment_sum_vec_kernel(
    const float* __restrict__ values, const int64_t* __restrict__ offsets,
    const int64_t* __restrict__ order, float* __restrict__ out, int64_t segments, int64_t width,
    int64_t value_rows, int* bad) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kGraphThreads / 32);
  const int64_t w4 = width / 4;
  for (int64_t s = static_cast<int64_t>(blockIdx.x) * (kGraphThreads / 32) + (threadIdx.x >> 5);
       s < segments; s += warps) {
    int64_t e0 = __ldg(offsets + s), e1 = __ldg(offsets + s + 1);
    if (e0 < 0 || e1 < e0 || e1 > value_rows) {
      // not a CSR range of the value / order rows: flag it, sum nothing
      if (lane == 0) atomicExch(bad, 1);
      e0 = e1 = 0;
    }
    float4* d4 = reinterpret_cast<float4*>(out + s * width);
    for (int64_t cb = 0; cb < w4; cb += 32 * kSegCols) {
      float4 acc[kSegCols];
#pragma unroll
      for (int k = 0; k < kSegCols; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int64_t eb = e0; eb < e1; eb += 32) {
        const int n = e1 - eb < 32 ? static_cast<int>(e1 - eb) : 32;
        int64_t mine = -1;
        if (lane < n) {
          const int64_t r = order ? __ldg(order + eb + lane) : eb + lane;
          if (r >= 0 && r < value_rows) mine = r;
          else if (cb == 0) atomicExch(bad, 1);
        }
        for (int j = 0; j < n; ++j) {
          const int64_t r = __shfl_sync(0xffffffffu, mine, j);
          if (r < 0) continue;
          const float4* row = reinterpret_cast<const float4*>(values + r * width);
          float4 v[kSegCols];
#pragma unroll
          for (int k = 0; k < kSegCols; ++k) {
            const int64_t c = cb + lane + 32 * k;
            v[k] = c < w4 ? __ldg(row + c) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int k = 0; k < kSegCols; ++k) {
            acc[k].x += v[k].x; acc[k].y += v[k].y; acc[k].z += v[k].z; acc[k].w += v[k].w;
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kSegCols; ++k) {
        const int64_t c = cb + lane + 32 * k;
        if (c < w4) d4[c] = acc[k];
      }
    }
  }
}

__global__ void __launch_bounds__(kGraphThreads) segment_sum_kernel(
    const float* __restrict__ values, const int64_t* __restrict__ offsets,
    const int64_t* __restrict__ order, float* __restrict__ out, int64_t segments, int64_t width,
    int64_t value_rows, bool vec, int* bad) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kGraphThreads / 32);
  for (int64_t s = static_cast<int64_t>(blockIdx.x) * (kGraphThreads / 32) + (threadIdx.x >> 5);
       s < segments; s += warps) {
    int64_t e0 = __ldg(offsets + s), e1 = __ldg(offsets + s + 1);
    float* dst = out + s * width;
    if (e0 < 0 || e1 < e0 || e1 > value_rows) {
      // not a CSR range of the value / order rows: flag it, sum nothing
      if (lane == 0) atomicExch(bad, 1);
      e0 = e1 = 0;
    }
    if (vec) {
      float4* d4 = reinterpret_cast<float4*>(dst);
      for (int64_t c = lane; c < width / 4; c += 32) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int64_t e = e0; e < e1; ++e) {
          const int64_t r = order ? __ldg(order + e) : e;
          if (r < 0 || r >= value_rows) {
            if (c == lane) atomicExch(bad, 1);
            continue;
          }
          const float4 v = __ldg(reinterpret_cast<const float4*>(values + r * width) + c);
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        d4[c] = acc;
      }
    } else {
      for (int64_t c = lane; c < width; c += 32) {
        float acc = 0.f;
        for (int64_t e = e0; e < e1; ++e) {
          const int64_t r = order ? __ldg(order + e) : e;
          if (r < 0 || r >= value_rows) {
            if (c == lane) atomicExch(bad, 1);
            continue;
          }
          acc += __ldg(values + r * width + c);
        }
        dst[c] = acc;
      }
    }
  }
}

// Flag set by a kernel that met an out-of-range row index (one per device).
__device__ int g_graph_bad_index;

int graph_grid(int64_t rows) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) device = 0;
  const int64_t warps_per_block = kGraphThreads / 32;
  int64_t blocks = (rows + warps_per_block - 1) / warps_per_block;
  const int64_t cap = static_cast<int64_t>(sm_count(device)) * 8;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

int* bad_flag() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_graph_bad_index) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

}  // namespace
}  // namespace ictc

using namespace ictc;

extern "C" int32_t ictc_o2_gather_rows(const float* source, const int64_t* index, float* out,
                                       int64_t rows, int64_t width, int64_t source_rows,
                                       void* stream) {
  if (rows < 0 || width < 0 || source_rows < 0)
    return fail(ICTC_ERR_INVALID, "rows, width and source_rows must be >= 0");
  if (rows == 0 || width == 0) return ICTC_OK;
  if (!source || !index || !out) return fail(ICTC_ERR_INVALID, "null pointer");
  int* bad = bad_flag();
  if (!bad) return fail(ICTC_ERR_CUDA, "device flag lookup failed");
  const bool vec = width % 4 == 0 && aligned(source, 16) && aligned(out, 16);
  gather_rows_kernel<<<graph_grid(rows), kGraphThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      source, index, out, rows, width, source_rows, vec, bad);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "gather_rows launch");
}

extern "C" int32_t ictc_o2_segment_sum(const float* values, const int64_t* offsets,
                                       const int64_t* order, float* out, int64_t segments,
                                       int64_t width, int64_t value_rows, void* stream) {
  if (segments < 0 || width < 0 || value_rows < 0)
    return fail(ICTC_ERR_INVALID, "segments, width and value_rows must be >= 0");
  if (segments == 0 || width == 0) return ICTC_OK;
  if (!offsets || !out || (value_rows > 0 && !values))
    return fail(ICTC_ERR_INVALID, "null pointer");
  int* bad = bad_flag();
  if (!bad) return fail(ICTC_ERR_CUDA, "device flag lookup failed");
  const bool vec = width % 4 == 0 && (value_rows == 0 || aligned(values, 16)) && aligned(out, 16);
  if (vec)
    segment_sum_vec_kernel<<<graph_grid(segments), kGraphThreads, 0,
                             static_cast<cudaStream_t>(stream)>>>(values, offsets, order, out,
                                                                  segments, width, value_rows,
                                                                  bad);
  else
    segment_sum_kernel<<<graph_grid(segments), kGraphThreads, 0,
                         static_cast<cudaStream_t>(stream)>>>(values, offsets, order, out,
                                                              segments, width, value_rows, false,
                                                              bad);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "segment_sum launch");
}

extern "C" int32_t ictc_o2_graph_bad_index(int32_t* flag) {
  if (!flag) return fail(ICTC_ERR_INVALID, "null output");
  int* bad = bad_flag();
  if (!bad) return fail(ICTC_ERR_CUDA, "device flag lookup failed");
  int host = 0;
  cudaError_t e = cudaMemcpy(&host, bad, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "graph flag read");
  const int zero = 0;
  e = cudaMemcpy(bad, &zero, sizeof(int), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "graph flag clear");
  *flag = host;
  return ICTC_OK;
}
