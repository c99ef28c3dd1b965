// FP32 uvu O(2) product (UvuTensorProduct) forward and VJP for sm_100a.
//
// Reference math (src/ictc_o2_hp/uvu_o2.py:50-73, uvu_triton.py:90-232):
//   proj_p[r,u,b] = sum_v w_p[u,v] y_j[r,v,b]
//   out_k[r,u,kc] += sum_{a,b} c_p[kc,a,b] x_i[r,u,a] proj_p[r,u,b]
// and its adjoints dx (same GEMM, g instead of x), dy (a GEMM over u) and dw (a GEMM
// over rows).  Three reduction axes, so three kernel shapes for shared weights:
//   * rowtile: 32 rows x 128 u per CTA, 4 rows x 4 u per thread; the weights of one
//     path (transposed to [v][u]) stream through a cp.async double buffer and
//     are reused over 32 rows; y of the 32 rows stays in shared memory.  Runs the
//     forward (paths grouped by output entry) and dx (grouped by first entry).
//   * dy tile: 32 rows x 32 v per CTA, four u-groups split the reduction over u
//     and are summed in a fixed order.
//   * dw tile: one path x 128 u x 32 v per CTA, reducing over all its rows (or a
//     fixed row chunk, then a fixed-order sum of chunks) — no atomics anywhere.
// Per-row weights (shared_weights=False) are pure streaming: one CTA per row,
// one thread per u, weights read once, weight gradients written once.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "rowtile.cuh"
#include "tma.cuh"
#include "uvu_table.cuh"

namespace ictc {

namespace {

UvuDev uvu_dev(const void* table, const UvuLayout& l) {
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

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------ shared weights

// wt[p][v][u] (u padded to Up) <- w[p][u][v]
__global__ void transpose_weights(const float* __restrict__ w, float* __restrict__ wt, int P,
                                  int U, int Up, int V) {
  const int64_t total = static_cast<int64_t>(P) * V * Up;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int u = static_cast<int>(idx % Up);
    const int64_t pv = idx / Up;
    const int v = static_cast<int>(pv % V);
    const int64_t p = pv / V;
    wt[idx] = u < U ? w[(p * U + u) * V + v] : 0.0f;
  }
}

constexpr int kDpStride = 68;  // floats per u in the dproj tile: 32 rows x 2 + pad

// dproj[u][r][b] = sum_{kc,a} c[kc][a][b] g_k[r,u,kc] x_i[r,u,a] for a 32-row x
// 128-u tile, written to shared memory by the whole CTA.
__device__ __forceinline__ void fill_dproj(float* dp, const float* __restrict__ x,
                                           const float* __restrict__ g, int64_t row0,
                                           int64_t rows, int ub, int U, int W1, int2 ei,
                                           int2 ek, const float* c) {
  for (int s = 0; s < 16; ++s) {
    const int q = threadIdx.x + s * 256;
    const int uu = q & 127, r = q >> 7;
    const int u = ub + uu;
    const int64_t row = row0 + r;
    float d0 = 0.f, d1 = 0.f;
    if (row < rows && u < U) {
      const float* xs = x + row * W1 + ei.x + u * ei.y;
      const float* gs = g + row * W1 + ek.x + u * ek.y;
      const float x0 = __ldg(xs), x1 = ei.y == 2 ? __ldg(xs + 1) : 0.f;
      const float g0 = __ldg(gs), g1 = ek.y == 2 ? __ldg(gs + 1) : 0.f;
      // dproj[b] = sum c[kc][a][b] g[kc] x[a]
      d0 = c[0] * g0 * x0 + c[2] * g0 * x1 + c[4] * g1 * x0 + c[6] * g1 * x1;
      d1 = c[1] * g0 * x0 + c[3] * g0 * x1 + c[5] * g1 * x0 + c[7] * g1 * x1;
    }
    dp[uu * kDpStride + 2 * r] = d0;
    dp[uu * kDpStride + 2 * r + 1] = d1;
  }
}

// dy_j[r,v,b] = sum_{p: j} sum_u w_p[u,v] dproj_p[r,u,b]; grid (row tiles, v tiles).
__global__ void __launch_bounds__(256)
    uvu_dy_tile(const float* __restrict__ x, const float* __restrict__ g,
                const float* __restrict__ w, float* __restrict__ dy, int64_t rows, int U, int V,
                int W1, int W2, UvuDev t, bool wvec) {
  extern __shared__ __align__(16) float sm[];
  float* dp = sm;  // [128 u][kDpStride]
  const int ug = threadIdx.x >> 6, t64 = threadIdx.x & 63;
  const int rq = t64 >> 3, vq = t64 & 7;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRT;
  const int v0 = blockIdx.y * 32 + vq * 4;
  float acc[4][4][2];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[r][q][0] = acc[r][q][1] = 0.f;
  for (int pos = 0; pos < t.np; ++pos) {
    const int p = t.by_j[pos];
    const int4 pt = t.paths[p];
    float c[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) c[e] = __ldg(t.coef + 8 * p + e);
    const int2 ei = t.in1[pt.x], ek = t.in1[pt.z];
    for (int ub = 0; ub < U; ub += 128) {
      __syncthreads();
      fill_dproj(dp, x, g, row0, rows, ub, U, W1, ei, ek, c);
      __syncthreads();
      const float* wp = w + static_cast<int64_t>(p) * U * V;
      for (int uu = ug * 32; uu < ug * 32 + 32; ++uu) {
        const int u = ub + uu;
        if (u >= U) break;
        float wv[4];
        if (wvec && v0 + 3 < V) {
          const float4 w4 = __ldg(reinterpret_cast<const float4*>(wp + static_cast<int64_t>(u) * V + v0));
          wv[0] = w4.x; wv[1] = w4.y; wv[2] = w4.z; wv[3] = w4.w;
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            wv[q] = v0 + q < V ? __ldg(wp + static_cast<int64_t>(u) * V + v0 + q) : 0.f;
        }
        const float4 d01 = *reinterpret_cast<const float4*>(dp + uu * kDpStride + rq * 8);
        const float4 d23 = *reinterpret_cast<const float4*>(dp + uu * kDpStride + rq * 8 + 4);
        const float d[4][2] = {{d01.x, d01.y}, {d01.z, d01.w}, {d23.x, d23.y}, {d23.z, d23.w}};
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[r][q][0] = fmaf(d[r][0], wv[q], acc[r][q][0]);
            acc[r][q][1] = fmaf(d[r][1], wv[q], acc[r][q][1]);
          }
      }
    }
    const bool last = pos + 1 == t.np || t.paths[t.by_j[pos + 1]].y != pt.y;
    if (last) {
      // fixed-order sum of the four u-groups, then store dy_j
      __syncthreads();
      float* red = sm;  // [4 groups][64 threads][32]
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          red[(ug * 64 + t64) * 32 + (r * 4 + q) * 2] = acc[r][q][0];
          red[(ug * 64 + t64) * 32 + (r * 4 + q) * 2 + 1] = acc[r][q][1];
          acc[r][q][0] = acc[r][q][1] = 0.f;
        }
      __syncthreads();
      if (ug == 0) {
        const int2 ej = t.in2[pt.y];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int64_t row = row0 + rq * 4 + r;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int v = v0 + q;
            float s0 = 0.f, s1 = 0.f;
            for (int gi = 0; gi < 4; ++gi) {
              s0 += red[(gi * 64 + t64) * 32 + (r * 4 + q) * 2];
              s1 += red[(gi * 64 + t64) * 32 + (r * 4 + q) * 2 + 1];
            }
            if (row < rows && v < V) {
              float* dst = dy + row * W2 + ej.x + v * ej.y;
              dst[0] = s0;
              if (ej.y == 2) dst[1] = s1;
            }
          }
        }
      }
    }
  }
}

// dw_p[u,v] (partial over a row chunk) = sum_{r,b} dproj_p[r,u,b] y_j[r,v,b].
// grid (paths, u tiles x v tiles, row chunks).
__global__ void __launch_bounds__(256)
    uvu_dw_tile(const float* __restrict__ x, const float* __restrict__ y,
                const float* __restrict__ g, float* __restrict__ dst, int64_t rows,
                int64_t chunk_rows, int64_t numel, int U, int V, int W1, int W2, UvuDev t) {
  extern __shared__ __align__(16) float sm[];
  float* dp = sm;                   // [32 rows][2 b][128 u]
  float* yt = sm + kRT * 2 * 128;   // [32 rows][2 b][32 v]
  const int p = blockIdx.x;
  const int ntu = (U + 127) / 128;
  const int ub = (blockIdx.y % ntu) * 128, vb = (blockIdx.y / ntu) * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int uq = (warp & 3) * 8 + (lane & 7);
  const int vq = (warp >> 2) * 4 + (lane >> 3);
  const int u0 = ub + uq * 4, v0 = vb + vq * 4;
  const int4 pt = t.paths[p];
  float c[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) c[e] = __ldg(t.coef + 8 * p + e);
  const int2 ei = t.in1[pt.x], ej = t.in2[pt.y], ek = t.in1[pt.z];
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
  const int64_t rbeg = static_cast<int64_t>(blockIdx.z) * chunk_rows;
  const int64_t rend = rbeg + chunk_rows < rows ? rbeg + chunk_rows : rows;
  for (int64_t row0 = rbeg; row0 < rend; row0 += kRT) {
    __syncthreads();
    for (int s = 0; s < 16; ++s) {
      const int q = threadIdx.x + s * 256;
      const int uu = q & 127, r = q >> 7;
      const int u = ub + uu;
      const int64_t row = row0 + r;
      float d0 = 0.f, d1 = 0.f;
      if (row < rend && u < U) {
        const float* xs = x + row * W1 + ei.x + u * ei.y;
        const float* gs = g + row * W1 + ek.x + u * ek.y;
        const float x0 = __ldg(xs), x1 = ei.y == 2 ? __ldg(xs + 1) : 0.f;
        const float g0 = __ldg(gs), g1 = ek.y == 2 ? __ldg(gs + 1) : 0.f;
        d0 = c[0] * g0 * x0 + c[2] * g0 * x1 + c[4] * g1 * x0 + c[6] * g1 * x1;
        d1 = c[1] * g0 * x0 + c[3] * g0 * x1 + c[5] * g1 * x0 + c[7] * g1 * x1;
      }
      dp[(r * 2) * 128 + uu] = d0;
      dp[(r * 2 + 1) * 128 + uu] = d1;
    }
    for (int q = threadIdx.x; q < kRT * 2 * 32; q += 256) {
      const int vv = q & 31, b = (q >> 5) & 1, r = q >> 6;
      const int v = vb + vv;
      const int64_t row = row0 + r;
      yt[q] = (row < rend && v < V && b < ej.y) ? __ldg(y + row * W2 + ej.x + v * ej.y + b) : 0.f;
    }
    __syncthreads();
    const int nb = ej.y;
    for (int r = 0; r < kRT; ++r) {
      for (int b = 0; b < nb; ++b) {
        const float4 d4 = *reinterpret_cast<const float4*>(dp + (r * 2 + b) * 128 + uq * 4);
        const float4 y4 = *reinterpret_cast<const float4*>(yt + (r * 2 + b) * 32 + vq * 4);
        const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
        const float yv[4] = {y4.x, y4.y, y4.z, y4.w};
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int bb = 0; bb < 4; ++bb) acc[a][bb] = fmaf(dv[a], yv[bb], acc[a][bb]);
      }
    }
  }
  float* out = dst + static_cast<int64_t>(blockIdx.z) * numel + static_cast<int64_t>(p) * U * V;
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int u = u0 + a, v = v0 + b;
      if (u < U && v < V) out[static_cast<int64_t>(u) * V + v] = acc[a][b];
    }
}

#include "uvu_tile.cuh"
#include "uvu_rowstream.cuh"
#include "uvu_rowquad.cuh"
#include "uvu_dy.cuh"
#include "uvu_dw.cuh"

// dst[i] = sum over chunks (fixed order) of partial[chunk][i].
__global__ void sum_chunks(const float* __restrict__ partial, float* __restrict__ dst,
                           int64_t numel, int chunks) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < numel;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < chunks; ++k) s += partial[static_cast<int64_t>(k) * numel + i];
    dst[i] = s;
  }
}

// ------------------------------------------------------------ per-row weights
//
// One CTA per row (grid-stride), thread u.  Per-thread operand slots live in
// shared memory, indexed by entry: slot (e, comp) of thread u at [(2e+comp) * bd + u].

__global__ void uvu_fwd_rowwise(const float* __restrict__ x, const float* __restrict__ y,
                                const float* __restrict__ w, float* __restrict__ out,
                                int64_t rows, int U, int V, int W1, int W2, int64_t Wn,
                                UvuDev t) {
  extern __shared__ __align__(16) float sm[];
  const int bd = blockDim.x, u = threadIdx.x;
  float* ys = sm;                              // [W2]
  float* xs = sm + ((W2 + 3) & ~3);            // [2 n1][bd]
  float* os = xs + 2 * t.n1 * bd;              // [2 n1][bd]
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    __syncthreads();
    for (int c = u; c < W2; c += bd) ys[c] = __ldg(y + row * W2 + c);
    for (int e = 0; e < t.n1; ++e) {
      const int2 en = t.in1[e];
      float v0 = 0.f, v1 = 0.f;
      if (u < U) {
        v0 = __ldg(x + row * W1 + en.x + u * en.y);
        v1 = en.y == 2 ? __ldg(x + row * W1 + en.x + u * en.y + 1) : 0.f;
      }
      xs[(2 * e) * bd + u] = v0;
      xs[(2 * e + 1) * bd + u] = v1;
      os[(2 * e) * bd + u] = 0.f;
      os[(2 * e + 1) * bd + u] = 0.f;
    }
    __syncthreads();
    if (u < U) {
      for (int p = 0; p < t.np; ++p) {
        const int4 pt = t.paths[p];
        const int2 ej = t.in2[pt.y];
        const float* wr = w + row * Wn + (static_cast<int64_t>(p) * U + u) * V;
        float p0 = 0.f, p1 = 0.f;
        for (int v = 0; v < V; ++v) {
          const float wv = __ldg(wr + v);
          p0 = fmaf(wv, ys[ej.x + v * ej.y], p0);
          if (ej.y == 2) p1 = fmaf(wv, ys[ej.x + v * ej.y + 1], p1);
        }
        const float* c = t.coef + 8 * p;
        const float x0 = xs[(2 * pt.x) * bd + u], x1 = xs[(2 * pt.x + 1) * bd + u];
        os[(2 * pt.z) * bd + u] +=
            __ldg(c) * x0 * p0 + __ldg(c + 1) * x0 * p1 + __ldg(c + 2) * x1 * p0 + __ldg(c + 3) * x1 * p1;
        os[(2 * pt.z + 1) * bd + u] +=
            __ldg(c + 4) * x0 * p0 + __ldg(c + 5) * x0 * p1 + __ldg(c + 6) * x1 * p0 + __ldg(c + 7) * x1 * p1;
      }
      for (int e = 0; e < t.n1; ++e) {
        const int2 en = t.in1[e];
        out[row * W1 + en.x + u * en.y] = os[(2 * e) * bd + u];
        if (en.y == 2) out[row * W1 + en.x + u * en.y + 1] = os[(2 * e + 1) * bd + u];
      }
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void uvu_bwd_rowwise(const float* __restrict__ x, const float* __restrict__ y,
                                const float* __restrict__ w, const float* __restrict__ g,
                                float* __restrict__ dx, float* __restrict__ dy,
                                float* __restrict__ dw, int64_t rows, int U, int V, int W1,
                                int W2, int64_t Wn, int needed, UvuDev t) {
  extern __shared__ __align__(16) float sm[];
  const int bd = blockDim.x, u = threadIdx.x;
  const int nw = bd >> 5, warp = u >> 5, lane = u & 31;
  const int W2a = (W2 + 3) & ~3;
  float* ys = sm;                        // [W2]
  float* xs = ys + W2a;                  // [2 n1][bd]
  float* gs = xs + 2 * t.n1 * bd;        // [2 n1][bd]
  float* ds = gs + 2 * t.n1 * bd;        // [2 n1][bd]  dx slots
  float* yp = ds + 2 * t.n1 * bd;        // [nw][W2a]   dy partial per warp
  const bool want_dx = needed & 1, want_dy = needed & 2, want_dw = needed & 4;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    __syncthreads();
    for (int c = u; c < W2; c += bd) ys[c] = __ldg(y + row * W2 + c);
    for (int c = u; c < nw * W2a; c += bd) yp[c] = 0.f;
    for (int e = 0; e < t.n1; ++e) {
      const int2 en = t.in1[e];
      float x0 = 0.f, x1 = 0.f, g0 = 0.f, g1 = 0.f;
      if (u < U) {
        const int64_t o = row * W1 + en.x + u * en.y;
        x0 = __ldg(x + o);
        g0 = __ldg(g + o);
        if (en.y == 2) {
          x1 = __ldg(x + o + 1);
          g1 = __ldg(g + o + 1);
        }
      }
      xs[(2 * e) * bd + u] = x0;
      xs[(2 * e + 1) * bd + u] = x1;
      gs[(2 * e) * bd + u] = g0;
      gs[(2 * e + 1) * bd + u] = g1;
      ds[(2 * e) * bd + u] = 0.f;
      ds[(2 * e + 1) * bd + u] = 0.f;
    }
    __syncthreads();
    const bool act = u < U;
    for (int p = 0; p < t.np; ++p) {
      const int4 pt = t.paths[p];
      const int2 ej = t.in2[pt.y];
      const float* c = t.coef + 8 * p;
      float cc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) cc[e] = __ldg(c + e);
      const float x0 = xs[(2 * pt.x) * bd + u], x1 = xs[(2 * pt.x + 1) * bd + u];
      const float g0 = gs[(2 * pt.z) * bd + u], g1 = gs[(2 * pt.z + 1) * bd + u];
      // dproj[b] = sum c[kc][a][b] g[kc] x[a]
      const float q0 = cc[0] * g0 * x0 + cc[2] * g0 * x1 + cc[4] * g1 * x0 + cc[6] * g1 * x1;
      const float q1 = cc[1] * g0 * x0 + cc[3] * g0 * x1 + cc[5] * g1 * x0 + cc[7] * g1 * x1;
      const int64_t wo = row * Wn + (static_cast<int64_t>(p) * U + (act ? u : 0)) * V;
      float p0 = 0.f, p1 = 0.f;
      for (int v = 0; v < V; ++v) {
        const float wv = act ? __ldg(w + wo + v) : 0.f;
        const float y0 = ys[ej.x + v * ej.y];
        const float y1 = ej.y == 2 ? ys[ej.x + v * ej.y + 1] : 0.f;
        p0 = fmaf(wv, y0, p0);
        p1 = fmaf(wv, y1, p1);
        if (want_dw && act) dw[wo + v] = q0 * y0 + q1 * y1;
        if (want_dy) {
          const float s0 = warp_sum(wv * q0);
          const float s1 = ej.y == 2 ? warp_sum(wv * q1) : 0.f;
          if (lane == 0) {
            yp[warp * W2a + ej.x + v * ej.y] += s0;
            if (ej.y == 2) yp[warp * W2a + ej.x + v * ej.y + 1] += s1;
          }
        }
      }
      if (want_dx && act) {  // dx[a] += c[kc][a][b] g[kc] p[b]
        ds[(2 * pt.x) * bd + u] += cc[0] * g0 * p0 + cc[1] * g0 * p1 + cc[4] * g1 * p0 + cc[5] * g1 * p1;
        ds[(2 * pt.x + 1) * bd + u] +=
            cc[2] * g0 * p0 + cc[3] * g0 * p1 + cc[6] * g1 * p0 + cc[7] * g1 * p1;
      }
    }
    __syncthreads();
    if (want_dx && act) {
      for (int e = 0; e < t.n1; ++e) {
        const int2 en = t.in1[e];
        dx[row * W1 + en.x + u * en.y] = ds[(2 * e) * bd + u];
        if (en.y == 2) dx[row * W1 + en.x + u * en.y + 1] = ds[(2 * e + 1) * bd + u];
      }
    }
    if (want_dy) {
      for (int c = u; c < W2; c += bd) {
        float s = 0.f;
        for (int k = 0; k < nw; ++k) s += yp[k * W2a + c];
        dy[row * W2 + c] = s;
      }
    }
  }
}

// ------------------------------------------------------------------ host side

struct UvuConfig {
  int U, V, m1, m2;
  bool full1, full2, component, path_norm;
};

int validate_uvu(const UvuConfig& c) {
  if (c.U < 1 || c.V < 1) return fail(ICTC_ERR_INVALID, "channels must be >= 1");
  if (c.m1 < 0 || c.m2 < 0) return fail(ICTC_ERR_INVALID, "m_max must be >= 0");
  if (c.m1 > 32 || c.m2 > 32) return fail(ICTC_ERR_UNSUPPORTED, "m_max above 32");
  if (c.U > 1024) return fail(ICTC_ERR_UNSUPPORTED, "channels above 1024");
  return ICTC_OK;
}

UvuConfig uvu_config(int32_t channels, int32_t channels_in2, int32_t m_max, int32_t parity,
                     int32_t m_max_in2, int32_t parity_in2, int32_t normalization,
                     int32_t path_normalization) {
  UvuConfig c;
  c.U = channels;
  c.V = channels_in2;
  c.m1 = m_max;
  c.m2 = m_max_in2;
  c.full1 = parity == ICTC_PARITY_FULL;
  c.full2 = parity_in2 == ICTC_PARITY_FULL;
  c.component = normalization == ICTC_NORM_COMPONENT;
  c.path_norm = path_normalization != 0;
  return c;
}

UvuTableH table_of(const UvuConfig& c) {
  return build_uvu_table(c.U, c.V, c.m1, c.full1, c.m2, c.full2, c.component, c.path_norm);
}

// Row chunks of the shared-weight dw: enough CTAs to fill the GPU, and no chunk
// longer than kDwChunkRows rows.  Each chunk's partial is a sequential FP32 sum of
// 2 x chunk rows terms per weight; at 65,536 rows per chunk the float64-normalised
// error of dw reached 1.4e-5 at 131,072 rows (the gate is 1e-5), at 1,024 rows it
// stays near 2e-6, and the chunk partials are summed in a fixed order after.
constexpr int64_t kDwChunkRows = 1024;

// Whether every second-input entry is read by some path (otherwise its gradient
// rows are never written by the dy kernels and are cleared first).
bool entries_all_used(const UvuTableH& t) {
  std::vector<char> used(t.in2.size(), 0);
  for (const UvuPathH& p : t.paths) used[p.j] = 1;
  for (char u : used)
    if (!u) return false;
  return true;
}

int64_t dw_chunks(int device, int64_t rows, int P, int U, int V) {
  const int64_t tiles = static_cast<int64_t>(P) * ((U + 127) / 128) * ((V + 31) / 32);
  int64_t chunks = (2 * sm_count(device) + tiles - 1) / tiles;
  const int64_t short_chunks = (rows + kDwChunkRows - 1) / kDwChunkRows;
  if (chunks < short_chunks) chunks = short_chunks;
  const int64_t max_chunks = (rows + 255) / 256;
  if (chunks > max_chunks) chunks = max_chunks;
  return chunks < 1 ? 1 : chunks;
}

}  // namespace

int uvu_take_device_error(int* code) {
  cudaError_t e;
  if (take_unit_device_error(code, &e) != 0) return cuda_fail(e, "uvu device error flag");
  return ICTC_OK;
}

}  // namespace ictc

using namespace ictc;

#define ICTC_UVU_CONFIG_ARGS                                                                   \
  int32_t channels, int32_t channels_in2, int32_t m_max, int32_t parity, int32_t m_max_in2,   \
      int32_t parity_in2, int32_t normalization, int32_t path_normalization

extern "C" int32_t ictc_o2_uvu_table(ICTC_UVU_CONFIG_ARGS, int32_t* table, int64_t capacity_words,
                                     int64_t* words) {
  if (words == nullptr) return fail(ICTC_ERR_INVALID, "words is null");
  const UvuConfig c = uvu_config(channels, channels_in2, m_max, parity, m_max_in2, parity_in2,
                                 normalization, path_normalization);
  int st = validate_uvu(c);
  if (st != ICTC_OK) return st;
  const UvuTableH t = table_of(c);
  const UvuLayout l = uvu_layout(static_cast<int>(t.in1.size()), static_cast<int>(t.in2.size()),
                                 static_cast<int>(t.paths.size()));
  *words = l.words;
  if (table == nullptr) return ICTC_OK;
  if (capacity_words < l.words) return fail(ICTC_ERR_INVALID, "table buffer too small");
  int32_t* w = table;
  std::memset(w, 0, static_cast<size_t>(l.words) * sizeof(int32_t));
  w[0] = l.n1; w[1] = l.n2; w[2] = l.np; w[3] = t.U; w[4] = t.V; w[5] = t.width1;
  w[6] = t.width2;
  w[8] = l.in1; w[9] = l.in2; w[10] = l.paths; w[11] = l.coef; w[12] = l.by_i; w[13] = l.by_j;
  w[14] = l.words;
  for (int e = 0; e < l.n1; ++e) {
    w[l.in1 + 2 * e] = t.in1[e].offset;
    w[l.in1 + 2 * e + 1] = t.in1[e].dim;
  }
  for (int e = 0; e < l.n2; ++e) {
    w[l.in2 + 2 * e] = t.in2[e].offset;
    w[l.in2 + 2 * e + 1] = t.in2[e].dim;
  }
  for (int p = 0; p < l.np; ++p) {
    w[l.paths + 4 * p] = t.paths[p].i;
    w[l.paths + 4 * p + 1] = t.paths[p].j;
    w[l.paths + 4 * p + 2] = t.paths[p].k;
    w[l.paths + 4 * p + 3] = 0;
    std::memcpy(w + l.coef + 8 * p, t.paths[p].c, 8 * sizeof(float));
    w[l.by_i + p] = t.by_i[p];
    w[l.by_j + p] = t.by_j[p];
  }
  return ICTC_OK;
}

extern "C" int32_t ictc_o2_uvu_workspace(ICTC_UVU_CONFIG_ARGS, int32_t shared, int64_t rows,
                                         int32_t device, size_t* forward_bytes,
                                         size_t* backward_bytes) {
  if (!forward_bytes || !backward_bytes) return fail(ICTC_ERR_INVALID, "null output");
  const UvuConfig c = uvu_config(channels, channels_in2, m_max, parity, m_max_in2, parity_in2,
                                 normalization, path_normalization);
  int st = validate_uvu(c);
  if (st != ICTC_OK) return st;
  if (rows < 0) return fail(ICTC_ERR_INVALID, "rows must be >= 0");
  const UvuTableH t = table_of(c);
  const int64_t P = static_cast<int64_t>(t.paths.size());
  const int Up = (c.U + 3) & ~3;
  if (!shared || rows == 0) {
    *forward_bytes = 0;
    *backward_bytes = 0;
    return ICTC_OK;
  }
  const size_t wt = static_cast<size_t>(P) * c.V * Up * sizeof(float);
  const int64_t chunks = dw_chunks(device, rows, static_cast<int>(P), c.U, c.V);
  const size_t partial =
      chunks > 1 ? static_cast<size_t>(chunks) * P * c.U * c.V * sizeof(float) : 0;
  *forward_bytes = wt;
  *backward_bytes = wt + partial;
  return ICTC_OK;
}

namespace {

int uvu_common(const UvuConfig& c, const void* table, int64_t rows, UvuTableH* t_out,
               UvuLayout* l_out) {
  int st = validate_uvu(c);
  if (st != ICTC_OK) return st;
  if (rows < 0) return fail(ICTC_ERR_INVALID, "rows must be >= 0");
  if (table == nullptr || !aligned(table, 16))
    return fail(ICTC_ERR_INVALID, "device table must be a 16-byte aligned device pointer");
  *t_out = table_of(c);
  *l_out = uvu_layout(static_cast<int>(t_out->in1.size()), static_cast<int>(t_out->in2.size()),
                      static_cast<int>(t_out->paths.size()));
  return ICTC_OK;
}

int rowwise_grid(int device, int64_t rows) {
  const int64_t cap = static_cast<int64_t>(sm_count(device)) * 16;
  return static_cast<int>(rows < cap ? rows : cap);
}

// Streams per-row weights with uvu_rowstream<MODE>; ICTC_ERR_UNSUPPORTED when the
// shape or alignment does not suit it (nothing launched).
template <int MODE>
int launch_rowstream(const RowStreamArgs& ra, int device, cudaStream_t s) {
  if (!rowstream_fits(ra.U, ra.V, ra.W1, ra.W2, ra.t.n1) || !aligned(ra.w, 16) ||
      (MODE == kRsBwd && (ra.needed & 4) && !aligned(ra.dw, 16)))
    return ICTC_ERR_UNSUPPORTED;
  const size_t smem = rowstream_smem(ra.U, ra.W2, ra.t.n1);
  const void* fn = reinterpret_cast<const void*>(&uvu_rowstream<MODE>);
  int st = allow_smem(fn, smem);
  if (st != ICTC_OK) return st;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kRsThreads, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  int64_t grid = static_cast<int64_t>(sm_count(device)) * (per_sm > 0 ? per_sm : 1);
  if (grid > ra.rows) grid = ra.rows;
  uvu_rowstream<MODE><<<static_cast<unsigned>(grid), kRsThreads, smem, s>>>(ra);
  e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "uvu row stream launch");
}

template <int MODE, int NQ, int R>
int launch_rowquad_shape(const RowStreamArgs& ra, int device, size_t smem, cudaStream_t s) {
  const void* fn = reinterpret_cast<const void*>(&uvu_rowquad<MODE, NQ, R>);
  int st = allow_smem(fn, smem);
  if (st != ICTC_OK) return st;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kRsThreads, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  int64_t grid = static_cast<int64_t>(sm_count(device)) * (per_sm > 0 ? per_sm : 1);
  if (grid > ra.rows) grid = ra.rows;
  uvu_rowquad<MODE, NQ, R><<<static_cast<unsigned>(grid), kRsThreads, smem, s>>>(ra);
  e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "uvu row quad launch");
}

template <int MODE, int NQ>
int launch_rowquad_nq(const RowStreamArgs& ra, int device, size_t smem, cudaStream_t s) {
  using Sh = RqShape<NQ>;
  const int r = rowquad_rows_per_lane<NQ>(ra.U);
  if (r == 1) return launch_rowquad_shape<MODE, NQ, 1>(ra, device, smem, s);
  if constexpr (Sh::L >= 2 && 2 * Sh::QT <= 4)
    if (r == 2) return launch_rowquad_shape<MODE, NQ, 2>(ra, device, smem, s);
  if constexpr (Sh::L >= 4 && Sh::QT == 1)
    if (r == 4) return launch_rowquad_shape<MODE, NQ, 4>(ra, device, smem, s);
  return ICTC_ERR_UNSUPPORTED;
}

// Per-row weights with uvu_rowquad<MODE> (V in {8, 16, 32, 64});
// ICTC_ERR_UNSUPPORTED when the shape or alignment does not suit it.
template <int MODE>
int launch_rowquad(const RowStreamArgs& ra, int device, cudaStream_t s) {
  if (!rowstream_fits(ra.U, ra.V, ra.W1, ra.W2, ra.t.n1) || !aligned(ra.w, 16) ||
      (MODE == kRsBwd && (ra.needed & 4) && !aligned(ra.dw, 16)))
    return ICTC_ERR_UNSUPPORTED;
  const size_t smem = rowquad_smem<MODE>(ra.U, ra.W2, ra.t.n1, ra.t.np);
  if (smem > 220 * 1024) return ICTC_ERR_UNSUPPORTED;
  switch (ra.V) {
    case 8: return launch_rowquad_nq<MODE, 2>(ra, device, smem, s);
    case 16: return launch_rowquad_nq<MODE, 4>(ra, device, smem, s);
    case 32: return launch_rowquad_nq<MODE, 8>(ra, device, smem, s);
    case 64: return launch_rowquad_nq<MODE, 16>(ra, device, smem, s);
    default: return ICTC_ERR_UNSUPPORTED;
  }
}

// Per-row-weight kernels in order of preference; ICTC_UVU_ROW_KERNEL = "quad",
// "stream" or "rowwise" starts the chain further down (tests cover each).
template <int MODE>
int launch_per_row(const RowStreamArgs& ra, int device, cudaStream_t s) {
  const char* pick = getenv("ICTC_UVU_ROW_KERNEL");
  const bool skip_quad = pick != nullptr && (strcmp(pick, "stream") == 0 || strcmp(pick, "rowwise") == 0);
  const bool skip_stream = pick != nullptr && strcmp(pick, "rowwise") == 0;
  int st = ICTC_ERR_UNSUPPORTED;
  if (!skip_quad) st = launch_rowquad<MODE>(ra, device, s);
  if (st == ICTC_ERR_UNSUPPORTED && !skip_stream) st = launch_rowstream<MODE>(ra, device, s);
  return st;
}

}  // namespace

extern "C" int32_t ictc_o2_uvu_forward(const float* left, const float* right, const float* weight,
                                       float* output, int64_t rows, ICTC_UVU_CONFIG_ARGS,
                                       int32_t shared, const void* device_table, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  const UvuConfig c = uvu_config(channels, channels_in2, m_max, parity, m_max_in2, parity_in2,
                                 normalization, path_normalization);
  UvuTableH th;
  UvuLayout l;
  int st = uvu_common(c, device_table, rows, &th, &l);
  if (st != ICTC_OK) return st;
  if (rows == 0) return ICTC_OK;
  if (!left || !right || !weight || !output) return fail(ICTC_ERR_INVALID, "null tensor pointer");
  const UvuDev t = uvu_dev(device_table, l);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const int W1 = th.width1, W2 = th.width2;
  const int64_t Wn = static_cast<int64_t>(l.np) * c.U * c.V;
  if (!shared) {
    RowStreamArgs ra{left, right, weight, nullptr, output, nullptr, nullptr, rows,
                     static_cast<int64_t>(l.np) * c.U * c.V, c.U, c.V, W1, W2, t, 0};
    st = launch_per_row<kRsFwd>(ra, device, s);
    if (st == ICTC_OK) return ICTC_OK;
    if (st != ICTC_ERR_UNSUPPORTED) return st;
    const int bd = ((c.U + 31) / 32) * 32;
    const size_t smem = (((W2 + 3) & ~3) + 4 * l.n1 * bd) * sizeof(float);
    if ((st = allow_smem(reinterpret_cast<const void*>(&uvu_fwd_rowwise), smem)) != ICTC_OK)
      return st;
    uvu_fwd_rowwise<<<rowwise_grid(device, rows), bd, smem, s>>>(left, right, weight, output,
                                                                 rows, c.U, c.V, W1, W2, Wn, t);
  } else {
    const int Up = (c.U + 3) & ~3;
    const size_t need = static_cast<size_t>(l.np) * c.V * Up * sizeof(float);
    if (workspace_bytes < need || (need && !workspace))
      return fail(ICTC_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, need);
    if (!aligned(workspace, 16)) return fail(ICTC_ERR_INVALID, "workspace must be 16-byte aligned");
    float* wt = static_cast<float*>(workspace);
    transpose_weights<<<1024, 256, 0, s>>>(weight, wt, l.np, c.U, Up, c.V);
    const bool vec = (W1 % 4 == 0) && (c.U % 4 == 0) && aligned(left, 16) && aligned(output, 16);
    UvuTileArgs ua{left, right, wt, output, rows, c.U, Up, c.V, W1, W2, t, vec};
    st = launch_uvu_tile<kUtFwd>(ua, s);
    if (st == ICTC_ERR_UNSUPPORTED) {  // second input too wide for the resident tile
      RowtileArgs ra{left, nullptr, right, nullptr, wt, nullptr, output, nullptr, rows,
                     c.U, Up, c.V, W1, W2, W2, t};
      st = launch_rowtile<kUvuFwd>(ra, s);
    }
    if (st != ICTC_OK) return st;
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "uvu forward launch");
}

extern "C" int32_t ictc_o2_uvu_backward(const float* left, const float* right, const float* weight,
                                        const float* grad_output, float* grad_left,
                                        float* grad_right, float* grad_weight, int64_t rows,
                                        ICTC_UVU_CONFIG_ARGS, int32_t shared, int32_t needed,
                                        const void* device_table, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  const UvuConfig c = uvu_config(channels, channels_in2, m_max, parity, m_max_in2, parity_in2,
                                 normalization, path_normalization);
  UvuTableH th;
  UvuLayout l;
  int st = uvu_common(c, device_table, rows, &th, &l);
  if (st != ICTC_OK) return st;
  if (needed < 0 || needed > 7) return fail(ICTC_ERR_INVALID, "needed must be a 3-bit mask");
  const int64_t Wn = static_cast<int64_t>(l.np) * c.U * c.V;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (rows == 0) {
    if ((needed & 4) && shared && grad_weight) {
      e = cudaMemsetAsync(grad_weight, 0, Wn * sizeof(float), s);
      if (e != cudaSuccess) return cuda_fail(e, "memset");
    }
    return ICTC_OK;
  }
  if (!left || !right || !weight || !grad_output) return fail(ICTC_ERR_INVALID, "null input");
  if (((needed & 1) && !grad_left) || ((needed & 2) && !grad_right) ||
      ((needed & 4) && !grad_weight))
    return fail(ICTC_ERR_INVALID, "null gradient output for a requested role");
  const UvuDev t = uvu_dev(device_table, l);
  int device = 0;
  e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const int W1 = th.width1, W2 = th.width2;
  if ((needed & 2) && !entries_all_used(th)) {
    // second-input entries that no path reads get a zero gradient
    e = cudaMemsetAsync(grad_right, 0, static_cast<size_t>(rows) * W2 * sizeof(float), s);
    if (e != cudaSuccess) return cuda_fail(e, "memset");
  }
  if (!shared) {
    RowStreamArgs ra{left, right, weight, grad_output, grad_left, grad_right, grad_weight, rows,
                     Wn, c.U, c.V, W1, W2, t, needed};
    st = launch_per_row<kRsBwd>(ra, device, s);
    if (st == ICTC_OK) return ICTC_OK;
    if (st != ICTC_ERR_UNSUPPORTED) return st;
    const int bd = ((c.U + 31) / 32) * 32;
    const int W2a = (W2 + 3) & ~3;
    const size_t smem = (W2a + 6 * l.n1 * bd + (bd / 32) * W2a) * sizeof(float);
    if (smem > 220 * 1024) return fail(ICTC_ERR_UNSUPPORTED, "row too wide for the rowwise VJP");
    if ((st = allow_smem(reinterpret_cast<const void*>(&uvu_bwd_rowwise), smem)) != ICTC_OK)
      return st;
    uvu_bwd_rowwise<<<rowwise_grid(device, rows), bd, smem, s>>>(
        left, right, weight, grad_output, grad_left, grad_right, grad_weight, rows, c.U, c.V, W1,
        W2, Wn, needed, t);
    e = cudaGetLastError();
    return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "uvu rowwise backward launch");
  }
  const int Up = (c.U + 3) & ~3;
  const size_t wt_bytes = static_cast<size_t>(l.np) * c.V * Up * sizeof(float);
  const int64_t chunks = dw_chunks(device, rows, l.np, c.U, c.V);
  const size_t part_bytes = chunks > 1 ? static_cast<size_t>(chunks) * Wn * sizeof(float) : 0;
  if (workspace_bytes < wt_bytes + part_bytes || !workspace)
    return fail(ICTC_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes,
                wt_bytes + part_bytes);
  if (!aligned(workspace, 16)) return fail(ICTC_ERR_INVALID, "workspace must be 16-byte aligned");
  float* wt = static_cast<float*>(workspace);
  float* partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + wt_bytes);
  if (needed & 1) {
    transpose_weights<<<1024, 256, 0, s>>>(weight, wt, l.np, c.U, Up, c.V);
    const bool vec = (W1 % 4 == 0) && (c.U % 4 == 0) && aligned(grad_output, 16) &&
                     aligned(grad_left, 16);
    UvuTileArgs ua{grad_output, right, wt, grad_left, rows, c.U, Up, c.V, W1, W2, t, vec};
    st = launch_uvu_tile<kUtDx>(ua, s);
    if (st == ICTC_ERR_UNSUPPORTED) {
      RowtileArgs ra{grad_output, nullptr, right, nullptr, wt, nullptr, grad_left, nullptr, rows,
                     c.U, Up, c.V, W1, W2, W2, t};
      st = launch_rowtile<kUvuDx>(ra, s);
    }
    if (st != ICTC_OK) return st;
  }
  if ((needed & 2) && uvu_dy_stage_fits(c.U, c.V, W1, aligned(left, 16) &&
                                                     aligned(grad_output, 16) &&
                                                     aligned(weight, 16)) &&
      uvu_dy_stage_smem(l.np) <= 227 * 1024) {
    const void* fn = reinterpret_cast<const void*>(&uvu_dy_stage);
    const size_t dy_smem = uvu_dy_stage_smem(l.np);
    if ((st = allow_smem(fn, dy_smem)) != ICTC_OK) return st;
    DyArgs da{left, grad_output, weight, grad_right, rows, c.U, c.V, W1, W2, t};
    uvu_dy_stage<<<static_cast<unsigned>(ceil_div(rows, kDyRows)), 256, dy_smem, s>>>(da);
  } else if (needed & 2) {
    const size_t smem = 128 * kDpStride * sizeof(float) > 4 * 64 * 32 * sizeof(float)
                            ? 128 * kDpStride * sizeof(float)
                            : 4 * 64 * 32 * sizeof(float);
    if ((st = allow_smem(reinterpret_cast<const void*>(&uvu_dy_tile), smem)) != ICTC_OK) return st;
    const bool wvec = (c.V % 4 == 0) && aligned(weight, 16);
    const dim3 grid(static_cast<unsigned>(ceil_div(rows, kRT)), (c.V + 31) / 32);
    uvu_dy_tile<<<grid, 256, smem, s>>>(left, grad_output, weight, grad_right, rows, c.U, c.V, W1,
                                        W2, t, wvec);
  }
  if ((needed & 4) && uvu_dw_stage_fits(c.U, c.V, W1, W2, aligned(left, 16) &&
                                                             aligned(right, 16) &&
                                                             aligned(grad_output, 16))) {
    const void* fn = reinterpret_cast<const void*>(&uvu_dw_stage);
    if ((st = allow_smem(fn, sizeof(DwSmem))) != ICTC_OK) return st;
    const int64_t chunk_rows = ((ceil_div(rows, chunks) + kDwRows - 1) / kDwRows) * kDwRows;
    float* dst = chunks > 1 ? partial : grad_weight;
    DwArgs wa{left, right, grad_output, dst, rows, chunk_rows, Wn, c.U, c.V, W1, W2, t};
    const dim3 grid(static_cast<unsigned>(l.np), static_cast<unsigned>(chunks));
    uvu_dw_stage<<<grid, 256, sizeof(DwSmem), s>>>(wa);
    if (chunks > 1) sum_chunks<<<1024, 256, 0, s>>>(partial, grad_weight, Wn, static_cast<int>(chunks));
  } else if (needed & 4) {
    const size_t smem = (kRT * 2 * 128 + kRT * 2 * 32) * sizeof(float);
    if ((st = allow_smem(reinterpret_cast<const void*>(&uvu_dw_tile), smem)) != ICTC_OK) return st;
    const int64_t chunk_rows = ((ceil_div(rows, chunks) + kRT - 1) / kRT) * kRT;
    const dim3 grid(static_cast<unsigned>(l.np), ((c.U + 127) / 128) * ((c.V + 31) / 32),
                    static_cast<unsigned>(chunks));
    float* dst = chunks > 1 ? partial : grad_weight;
    uvu_dw_tile<<<grid, 256, smem, s>>>(left, right, grad_output, dst, rows, chunk_rows, Wn, c.U,
                                        c.V, W1, W2, t);
    if (chunks > 1) sum_chunks<<<1024, 256, 0, s>>>(partial, grad_weight, Wn, static_cast<int>(chunks));
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "uvu backward launch");
}
