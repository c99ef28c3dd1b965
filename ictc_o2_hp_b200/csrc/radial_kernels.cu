// Radial-affine + V=1 uvu fusion (RadialUvuTensorProduct) for sm_100a.
//
// Reference: src/ictc_o2_hp/radial_uvu.py:21-66 and radial_streamed.py:37-139,
// docs/RADIAL.md: per edge e, path p and channel u
//   w[e,p,u] = sum_h hidden[e,h] alpha[p*U + u, h] + bias[p*U + u]
//   out_k[e,u,kc] += sum_{a,b} c_p[kc,a,b] x_i[e,u,a] y_j[e,b] w[e,p,u]
// The reference materialises w per 8192-edge block with cuBLAS.  Here the edge
// weights never reach HBM:
//   * forward and (dx, dy): rowtile<kRadFwd / kRadDx> regenerate w in registers
//     from a 32-edge hidden tile and streamed alpha blocks (rowtile.cuh);
//   * dhidden[e,h] = sum_{p,u} gw[e,p,u] alpha[p*U+u, h], gw = c g_k x_i y_j:
//     a row-tiled kernel that forms gw tiles in shared memory;
//   * dalpha[p*U+u, h] = sum_e gw[e,p,u] hidden[e,h] and dbias[p*U+u] = sum_e gw:
//     a path-tiled reduction over edges (fixed row chunks, fixed-order sum).
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "rowtile.cuh"
#include "uvu_table.cuh"

namespace ictc {

namespace {

UvuDev radial_dev(const void* table, const UvuLayout& l) {
  const int* w = static_cast<const int*>(table);
  UvuDev d;
  d.in1 = reinterpret_cast<const int2*>(w + l.in1);
  d.in2 = reinterpret_cast<const int2*>(w + l.in2);
  d.paths = reinterpret_cast<const int4*>(w + l.paths);
  d.coef = reinterpret_cast<const float*>(w + l.coef);
  d.by_i = w + l.by_i;
  d.by_j = w + l.by_j;
  d.n1 = l.n1;
  d.n2 = l.n2;
  d.np = l.np;
  return d;
}

// at[p][h][u] (u padded to Up) <- alpha[p*U + u][h]
__global__ void transpose_alpha(const float* __restrict__ a, float* __restrict__ at, int P, int U,
                                int Up, int H) {
  const int64_t total = static_cast<int64_t>(P) * H * Up;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int u = static_cast<int>(idx % Up);
    const int64_t ph = idx / Up;
    const int h = static_cast<int>(ph % H);
    const int64_t p = ph / H;
    at[idx] = u < U ? a[(p * U + u) * H + h] : 0.0f;
  }
}

// gw[r,u] = sum_{kc,a,b} c[kc,a,b] g_k[r,u,kc] x_i[r,u,a] y_j[r,b]
__device__ __forceinline__ float edge_weight_grad(const float* __restrict__ x,
                                                  const float* __restrict__ g, const float* yrow,
                                                  int64_t row, int u, int W1, int2 ei, int2 ek,
                                                  int2 ej, const float* c) {
  const float* xs = x + row * W1 + ei.x + u * ei.y;
  const float* gs = g + row * W1 + ek.x + u * ek.y;
  const float x0 = __ldg(xs), x1 = ei.y == 2 ? __ldg(xs + 1) : 0.f;
  const float g0 = __ldg(gs), g1 = ek.y == 2 ? __ldg(gs + 1) : 0.f;
  const float y0 = yrow[ej.x], y1 = ej.y == 2 ? yrow[ej.x + 1] : 0.f;
  const float t0 = c[0] * g0 * x0 + c[2] * g0 * x1 + c[4] * g1 * x0 + c[6] * g1 * x1;
  const float t1 = c[1] * g0 * x0 + c[3] * g0 * x1 + c[5] * g1 * x0 + c[7] * g1 * x1;
  return t0 * y0 + t1 * y1;
}

constexpr int kDhRows = 64;

// dhidden for 64 edges x 64 h per CTA (grid.y over h blocks): per path, the gw tile
// [u][64 edges] goes to shared memory, then dh[e,h] += sum_u gw[e,u] alpha[p*U+u,h].
__global__ void __launch_bounds__(256)
    radial_dhidden(const float* __restrict__ x, const float* __restrict__ ang,
                   const float* __restrict__ g, const float* __restrict__ alpha,
                   float* __restrict__ dh, int64_t rows, int U, int H, int W1, int W2, UvuDev t,
                   bool avec) {
  extern __shared__ __align__(16) float sm[];
  const int W2a = (W2 + 3) & ~3;
  float* angt = sm;                     // [64 rows][W2a]
  float* gwt = sm + kDhRows * W2a;      // [U][64 rows]
  const int rq = threadIdx.x >> 4, hq = threadIdx.x & 15;  // 16 x 16
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kDhRows;
  const int h0 = blockIdx.y * 64 + hq * 4;
  for (int idx = threadIdx.x; idx < kDhRows * W2; idx += blockDim.x) {
    const int r = idx / W2, col = idx % W2;
    const int64_t row = row0 + r;
    angt[r * W2a + col] = row < rows ? __ldg(ang + row * W2 + col) : 0.f;
  }
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
  for (int p = 0; p < t.np; ++p) {
    const int4 pt = t.paths[p];
    float c[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) c[e] = __ldg(t.coef + 8 * p + e);
    const int2 ei = t.in1[pt.x], ej = t.in2[pt.y], ek = t.in1[pt.z];
    __syncthreads();
    for (int q = threadIdx.x; q < kDhRows * U; q += blockDim.x) {
      const int u = q % U, r = q / U;
      const int64_t row = row0 + r;
      gwt[u * kDhRows + r] =
          row < rows ? edge_weight_grad(x, g, angt + r * W2a, row, u, W1, ei, ek, ej, c) : 0.f;
    }
    __syncthreads();
    const float* ap = alpha + static_cast<int64_t>(p) * U * H;
    for (int u = 0; u < U; ++u) {
      float av[4];
      if (avec && h0 + 3 < H) {
        const float4 a4 = __ldg(reinterpret_cast<const float4*>(ap + static_cast<int64_t>(u) * H + h0));
        av[0] = a4.x; av[1] = a4.y; av[2] = a4.z; av[3] = a4.w;
      } else {
#pragma unroll
        for (int b = 0; b < 4; ++b) av[b] = h0 + b < H ? __ldg(ap + static_cast<int64_t>(u) * H + h0 + b) : 0.f;
      }
      const float4 g4 = *reinterpret_cast<const float4*>(gwt + u * kDhRows + rq * 4);
      const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(gv[a], av[b], acc[a][b]);
    }
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t row = row0 + rq * 4 + a;
#pragma unroll
    for (int b = 0; b < 4; ++b)
      if (row < rows && h0 + b < H) dh[row * H + h0 + b] = acc[a][b];
  }
}

// dalpha[p*U + u, h] (and dbias) partial over a row chunk; grid (paths, u blocks x h
// blocks, chunks).  Tile 128 u x 32 h, thread 4 u x 4 h.
__global__ void __launch_bounds__(256)
    radial_dalpha(const float* __restrict__ x, const float* __restrict__ ang,
                  const float* __restrict__ g, const float* __restrict__ hidden,
                  float* __restrict__ da, float* __restrict__ db, int64_t rows,
                  int64_t chunk_rows, int64_t da_numel, int64_t db_numel, int U, int H, int W1,
                  int W2, UvuDev t) {
  extern __shared__ __align__(16) float sm[];
  float* gwt = sm;                // [32 rows][128 u]
  float* ht = sm + kRT * 128;     // [32 rows][32 h]
  const int p = blockIdx.x;
  const int ntu = (U + 127) / 128;
  const int ub = (blockIdx.y % ntu) * 128, hb = (blockIdx.y / ntu) * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int uq = (warp & 3) * 8 + (lane & 7);
  const int hq = (warp >> 2) * 4 + (lane >> 3);
  const int u0 = ub + uq * 4, h0 = hb + hq * 4;
  const int4 pt = t.paths[p];
  float c[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) c[e] = __ldg(t.coef + 8 * p + e);
  const int2 ei = t.in1[pt.x], ej = t.in2[pt.y], ek = t.in1[pt.z];
  float acc[4][4], bacc[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    bacc[a] = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
  }
  const int64_t rbeg = static_cast<int64_t>(blockIdx.z) * chunk_rows;
  const int64_t rend = rbeg + chunk_rows < rows ? rbeg + chunk_rows : rows;
  for (int64_t row0 = rbeg; row0 < rend; row0 += kRT) {
    __syncthreads();
    for (int s = 0; s < 16; ++s) {
      const int q = threadIdx.x + s * 256;
      const int uu = q & 127, r = q >> 7;
      const int u = ub + uu;
      const int64_t row = row0 + r;
      float v = 0.f;
      if (row < rend && u < U) {
        const float* ys = ang + row * W2 + ej.x;
        const float y0 = __ldg(ys), y1 = ej.y == 2 ? __ldg(ys + 1) : 0.f;
        const float* xs = x + row * W1 + ei.x + u * ei.y;
        const float* gs = g + row * W1 + ek.x + u * ek.y;
        const float x0 = __ldg(xs), x1 = ei.y == 2 ? __ldg(xs + 1) : 0.f;
        const float g0 = __ldg(gs), g1 = ek.y == 2 ? __ldg(gs + 1) : 0.f;
        const float t0 = c[0] * g0 * x0 + c[2] * g0 * x1 + c[4] * g1 * x0 + c[6] * g1 * x1;
        const float t1 = c[1] * g0 * x0 + c[3] * g0 * x1 + c[5] * g1 * x0 + c[7] * g1 * x1;
        v = t0 * y0 + t1 * y1;
      }
      gwt[r * 128 + uu] = v;
    }
    for (int q = threadIdx.x; q < kRT * 32; q += 256) {
      const int hh = q & 31, r = q >> 5;
      const int h = hb + hh;
      const int64_t row = row0 + r;
      ht[q] = (row < rend && h < H) ? __ldg(hidden + row * H + h) : 0.f;
    }
    __syncthreads();
    for (int r = 0; r < kRT; ++r) {
      const float4 g4 = *reinterpret_cast<const float4*>(gwt + r * 128 + uq * 4);
      const float4 h4 = *reinterpret_cast<const float4*>(ht + r * 32 + hq * 4);
      const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
      const float hv[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        bacc[a] += gv[a];
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(gv[a], hv[b], acc[a][b]);
      }
    }
  }
  float* dout = da + static_cast<int64_t>(blockIdx.z) * da_numel;
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int u = u0 + a, h = h0 + b;
      if (u < U && h < H) dout[(static_cast<int64_t>(p) * U + u) * H + h] = acc[a][b];
    }
  if (db != nullptr && hb == 0 && hq == 0) {
    float* bout = db + static_cast<int64_t>(blockIdx.z) * db_numel;
#pragma unroll
    for (int a = 0; a < 4; ++a)
      if (u0 + a < U) bout[static_cast<int64_t>(p) * U + u0 + a] = bacc[a];
  }
}

__global__ void radial_sum_chunks(const float* __restrict__ partial, float* __restrict__ dst,
                                  int64_t numel, int chunks) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < numel;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < chunks; ++k) s += partial[static_cast<int64_t>(k) * numel + i];
    dst[i] = s;
  }
}

struct RadialConfig {
  int U, M, H;
  bool full1, full2, component;
  int M2;
};

int radial_validate(const RadialConfig& c) {
  if (c.U < 1 || c.H < 1) return fail(ICTC_ERR_INVALID, "channels and hidden must be >= 1");
  if (c.M < 0 || c.M2 < 0) return fail(ICTC_ERR_INVALID, "m_max must be >= 0");
  if (c.U > kUT)
    return fail(ICTC_ERR_UNSUPPORTED, "radial fusion supports channels <= %d (got %d)", kUT, c.U);
  if (c.M > 32 || c.M2 > 32) return fail(ICTC_ERR_UNSUPPORTED, "m_max above 32");
  return ICTC_OK;
}

int64_t radial_chunks(int device, int64_t rows, int P, int U, int H) {
  const int64_t tiles = static_cast<int64_t>(P) * ((U + 127) / 128) * ((H + 31) / 32);
  int64_t chunks = (2 * sm_count(device) + tiles - 1) / tiles;
  const int64_t max_chunks = (rows + 255) / 256;
  if (chunks > max_chunks) chunks = max_chunks;
  return chunks < 1 ? 1 : chunks;
}

}  // namespace

}  // namespace ictc

using namespace ictc;

#define ICTC_RADIAL_ARGS                                                                     \
  int32_t channels, int32_t m_max, int32_t parity, int32_t m_max_in2, int32_t parity_in2,   \
      int32_t normalization, int32_t path_normalization, int32_t hidden

namespace {

int radial_setup(ICTC_RADIAL_ARGS, int64_t rows, const void* table, RadialConfig* c,
                 UvuTableH* th, UvuLayout* l) {
  c->U = channels;
  c->M = m_max;
  c->M2 = m_max_in2;
  c->H = hidden;
  c->full1 = parity == ICTC_PARITY_FULL;
  c->full2 = parity_in2 == ICTC_PARITY_FULL;
  c->component = normalization == ICTC_NORM_COMPONENT;
  int st = radial_validate(*c);
  if (st != ICTC_OK) return st;
  if (rows < 0) return fail(ICTC_ERR_INVALID, "rows must be >= 0");
  if (table == nullptr || !aligned(table, 16))
    return fail(ICTC_ERR_INVALID, "device table must be a 16-byte aligned device pointer");
  *th = build_uvu_table(c->U, 1, c->M, c->full1, c->M2, c->full2, c->component,
                        path_normalization != 0);
  *l = uvu_layout(static_cast<int>(th->in1.size()), static_cast<int>(th->in2.size()),
                  static_cast<int>(th->paths.size()));
  return ICTC_OK;
}

}  // namespace

extern "C" int32_t ictc_o2_radial_workspace(ICTC_RADIAL_ARGS, int64_t rows, int32_t device,
                                            size_t* forward_bytes, size_t* backward_bytes) {
  if (!forward_bytes || !backward_bytes) return fail(ICTC_ERR_INVALID, "null output");
  RadialConfig c{};
  c.U = channels; c.M = m_max; c.M2 = m_max_in2; c.H = hidden;
  c.full1 = parity == ICTC_PARITY_FULL; c.full2 = parity_in2 == ICTC_PARITY_FULL;
  c.component = normalization == ICTC_NORM_COMPONENT;
  int st = radial_validate(c);
  if (st != ICTC_OK) return st;
  const UvuTableH th = build_uvu_table(c.U, 1, c.M, c.full1, c.M2, c.full2, c.component,
                                       path_normalization != 0);
  const int64_t P = static_cast<int64_t>(th.paths.size());
  const int Up = (c.U + 3) & ~3;
  const size_t at = static_cast<size_t>(P) * c.H * Up * sizeof(float);
  if (rows <= 0) {
    *forward_bytes = 0;
    *backward_bytes = 0;
    return ICTC_OK;
  }
  const int64_t chunks = radial_chunks(device, rows, static_cast<int>(P), c.U, c.H);
  const size_t Wn = static_cast<size_t>(P) * c.U;
  const size_t part = chunks > 1 ? static_cast<size_t>(chunks) * (Wn * c.H + Wn) * sizeof(float) : 0;
  *forward_bytes = at;
  *backward_bytes = at + part;
  return ICTC_OK;
}

extern "C" int32_t ictc_o2_radial_forward(const float* left, const float* angular,
                                          const float* radial_hidden, const float* alpha,
                                          const float* bias, float* output, int64_t rows,
                                          ICTC_RADIAL_ARGS, const void* device_table,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  RadialConfig c{};
  UvuTableH th;
  UvuLayout l;
  int st = radial_setup(channels, m_max, parity, m_max_in2, parity_in2, normalization,
                        path_normalization, hidden, rows, device_table, &c, &th, &l);
  if (st != ICTC_OK) return st;
  if (rows == 0) return ICTC_OK;
  if (!left || !angular || !radial_hidden || !alpha || !output)
    return fail(ICTC_ERR_INVALID, "null tensor pointer");
  const int Up = (c.U + 3) & ~3;
  const size_t need = static_cast<size_t>(l.np) * c.H * Up * sizeof(float);
  if (workspace_bytes < need || !workspace || !aligned(workspace, 16))
    return fail(ICTC_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu (16-byte aligned)",
                workspace_bytes, need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* at = static_cast<float*>(workspace);
  transpose_alpha<<<1024, 256, 0, s>>>(alpha, at, l.np, c.U, Up, c.H);
  const size_t smem = rowtile_smem(kRadFwd, c.H, th.width2);
  if (smem > 220 * 1024) return fail(ICTC_ERR_UNSUPPORTED, "hidden width too large (%d)", c.H);
  if ((st = allow_smem(reinterpret_cast<const void*>(&rowtile<kRadFwd>), smem)) != ICTC_OK)
    return st;
  const UvuDev t = radial_dev(device_table, l);
  RowtileArgs ra{left, nullptr, radial_hidden, angular, at, bias, output, nullptr, rows,
                 c.U, Up, c.H, th.width1, c.H, th.width2, t};
  const dim3 grid(static_cast<unsigned>(ceil_div(rows, kRT)), 1);
  rowtile<kRadFwd><<<grid, 256, smem, s>>>(ra);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "radial forward launch");
}

extern "C" int32_t ictc_o2_radial_backward(
    const float* left, const float* angular, const float* radial_hidden, const float* alpha,
    const float* bias, const float* grad_output, float* grad_left, float* grad_angular,
    float* grad_hidden, float* grad_alpha, float* grad_bias, int64_t rows, ICTC_RADIAL_ARGS,
    int32_t needed, const void* device_table, void* workspace, size_t workspace_bytes,
    void* stream) {
  RadialConfig c{};
  UvuTableH th;
  UvuLayout l;
  int st = radial_setup(channels, m_max, parity, m_max_in2, parity_in2, normalization,
                        path_normalization, hidden, rows, device_table, &c, &th, &l);
  if (st != ICTC_OK) return st;
  if (needed < 0 || needed > 31) return fail(ICTC_ERR_INVALID, "needed must be a 5-bit mask");
  const int64_t Wn = static_cast<int64_t>(l.np) * c.U;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (rows == 0) {
    if ((needed & 8) && grad_alpha) {
      e = cudaMemsetAsync(grad_alpha, 0, Wn * c.H * sizeof(float), s);
      if (e != cudaSuccess) return cuda_fail(e, "memset");
    }
    if ((needed & 16) && grad_bias) {
      e = cudaMemsetAsync(grad_bias, 0, Wn * sizeof(float), s);
      if (e != cudaSuccess) return cuda_fail(e, "memset");
    }
    return ICTC_OK;
  }
  if (!left || !angular || !radial_hidden || !alpha || !grad_output)
    return fail(ICTC_ERR_INVALID, "null input");
  if (((needed & 1) && !grad_left) || ((needed & 2) && !grad_angular) ||
      ((needed & 4) && !grad_hidden) || ((needed & 8) && !grad_alpha) ||
      ((needed & 16) && !grad_bias))
    return fail(ICTC_ERR_INVALID, "null gradient output for a requested role");
  int device = 0;
  e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const int Up = (c.U + 3) & ~3;
  const size_t at_bytes = static_cast<size_t>(l.np) * c.H * Up * sizeof(float);
  const int64_t chunks = radial_chunks(device, rows, l.np, c.U, c.H);
  const size_t part_bytes =
      chunks > 1 ? static_cast<size_t>(chunks) * (Wn * c.H + Wn) * sizeof(float) : 0;
  if (workspace_bytes < at_bytes + part_bytes || !workspace || !aligned(workspace, 16))
    return fail(ICTC_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu (16-byte aligned)",
                workspace_bytes, at_bytes + part_bytes);
  const UvuDev t = radial_dev(device_table, l);
  const int W1 = th.width1, W2 = th.width2;
  float* at = static_cast<float*>(workspace);
  float* partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + at_bytes);
  if (needed & 3) {
    // dx and dy together: both need the regenerated edge weights
    transpose_alpha<<<1024, 256, 0, s>>>(alpha, at, l.np, c.U, Up, c.H);
    const size_t smem = rowtile_smem(kRadDx, c.H, W2);
    if (smem > 220 * 1024) return fail(ICTC_ERR_UNSUPPORTED, "hidden width too large (%d)", c.H);
    if ((st = allow_smem(reinterpret_cast<const void*>(&rowtile<kRadDx>), smem)) != ICTC_OK)
      return st;
    // scratch outputs when only one of dx / dy is requested are not allowed to
    // alias inputs; the caller passes both buffers (see the Python wrapper)
    if (!grad_left || !grad_angular)
      return fail(ICTC_ERR_INVALID, "dx and dy buffers are both required when either is");
    RowtileArgs ra{grad_output, left, radial_hidden, angular, at, bias, grad_left, grad_angular,
                   rows, c.U, Up, c.H, W1, c.H, W2, t};
    const dim3 grid(static_cast<unsigned>(ceil_div(rows, kRT)), 1);
    rowtile<kRadDx><<<grid, 256, smem, s>>>(ra);
  }
  if (needed & 4) {
    const int W2a = (W2 + 3) & ~3;
    const size_t smem = (static_cast<size_t>(kDhRows) * W2a + static_cast<size_t>(c.U) * kDhRows) *
                        sizeof(float);
    if ((st = allow_smem(reinterpret_cast<const void*>(&radial_dhidden), smem)) != ICTC_OK)
      return st;
    const bool avec = (c.H % 4 == 0) && aligned(alpha, 16);
    const dim3 grid(static_cast<unsigned>(ceil_div(rows, kDhRows)), (c.H + 63) / 64);
    radial_dhidden<<<grid, 256, smem, s>>>(left, angular, grad_output, alpha, grad_hidden, rows,
                                           c.U, c.H, W1, W2, t, avec);
  }
  if (needed & 24) {
    // grad_alpha doubles as scratch when only the bias gradient is requested
    if (!grad_alpha) return fail(ICTC_ERR_INVALID, "grad_alpha is required when dbias is");
    const size_t smem = (kRT * 128 + kRT * 32) * sizeof(float);
    if ((st = allow_smem(reinterpret_cast<const void*>(&radial_dalpha), smem)) != ICTC_OK)
      return st;
    const int64_t chunk_rows = ((ceil_div(rows, chunks) + kRT - 1) / kRT) * kRT;
    const dim3 grid(static_cast<unsigned>(l.np), ((c.U + 127) / 128) * ((c.H + 31) / 32),
                    static_cast<unsigned>(chunks));
    const int64_t da_numel = Wn * c.H;
    float* da = chunks > 1 ? partial : grad_alpha;
    float* db = chunks > 1 ? partial + chunks * da_numel : ((needed & 16) ? grad_bias : nullptr);
    radial_dalpha<<<grid, 256, smem, s>>>(left, angular, grad_output, radial_hidden, da, db, rows,
                                          chunk_rows, da_numel, Wn, c.U, c.H, W1, W2, t);
    if (chunks > 1) {
      radial_sum_chunks<<<1024, 256, 0, s>>>(partial, grad_alpha, da_numel,
                                             static_cast<int>(chunks));
      if (needed & 16)
        radial_sum_chunks<<<256, 256, 0, s>>>(partial + chunks * da_numel, grad_bias, Wn,
                                              static_cast<int>(chunks));
    }
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "radial backward launch");
}
