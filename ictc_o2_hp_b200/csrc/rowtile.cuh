// Row-tiled GEMM + O(2) coupling kernel shared by the uvu and radial products.
//
// A CTA owns RT rows x UT channels u (RT x UT = 4096: 32 x 128, or 64 x 64 for
// products with at most 64 channels; 256 threads, 4 rows x 4 u each) and walks
// the paths of the product.  Per path p it forms, for every (row, u),
//   proj[r, u, b] = sum_k A[r, k, b] * Wp[k, u]                       (a GEMM)
// where A is the second input y_j (uvu; k = v, b = component of entry j) or the
// radial hidden features (radial; k = h, one column), and Wp is the path's weight
// block ([k][u], streamed through a cp.async double buffer, so each weight is
// reused over 32 rows).  Then it couples proj with a per-(row, u) operand:
//   kUvuFwd / kRadFwd:  out_k[r,u,kc] += sum_{a,b} c[kc,a,b] x_i[r,u,a] q[b]
//   kUvuDx  / kRadDx:   dx_i[r,u,a]   += sum_{kc,b} c[kc,a,b] g_k[r,u,kc] q[b]
// with q = proj (uvu) or q[b] = (proj + bias_p[u]) * y_j[r, b] (radial: the edge
// weight w[r,p,u] regenerated in registers, times the angular entry).  kRadDx
// also accumulates dy_j[r, b] += sum_u sum c g_k x_i w, reduced over u inside the
// CTA in a fixed order.  Paths are visited grouped by the output slot (by k for
// the forward, by i for dx), so only one output tile is live in registers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace ictc {

enum RowMode { kUvuFwd = 0, kUvuDx = 1, kRadFwd = 2, kRadDx = 3 };

constexpr int kRT = 32;   // rows per CTA of the 128-channel tile
constexpr int kUT = 128;  // widest channel tile
constexpr int kKC = 32;   // k per weight tile

// Rows per CTA for a channel tile of UT (the tile holds 4096 (row, u) outputs).
template <int UT>
constexpr int rows_per_tile() { return 4096 / UT; }

// Odd row stride of the small per-row tiles (angular input, dy partials): lanes
// of one warp read eight rows at a stride of 4 rows, conflict-free when odd.
__host__ __device__ constexpr int odd_stride(int w) { return (w % 2 == 1) ? w : w + 1; }

struct UvuDev {
  const int2* in1;
  const int2* in2;
  const int4* paths;
  const float* coef;
  const int* by_i;
  const int* by_j;
  int n1, n2, np;
};

struct RowtileArgs {
  const float* opnd;   // x (forward modes) or g (dx modes), [rows, W1]
  const float* opnd2;  // x for kRadDx (dy needs both g and x)
  const float* a_src;  // GEMM A: y [rows, W2] (uvu) or hidden [rows, Wa] (radial)
  const float* ang;    // radial angular input [rows, W2]
  const float* wt;     // weight blocks [P][K][Up]
  const float* bias;   // radial bias [P * U] or nullptr
  float* out;          // forward output or dx, [rows, W1]
  float* dy;           // kRadDx: dy [rows, W2]
  int64_t rows;
  int U, Up, K, W1, Wa, W2;
  UvuDev t;
};

__device__ __forceinline__ void rt_cp_async16(void* smem, const void* gmem, bool valid) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(bytes)
               : "memory");
}

// Dynamic shared memory of rowtile<MODE, UT> for a given A width and W2.
inline size_t rowtile_smem(int mode, int ut, int Wa, int W2) {
  const size_t rt = static_cast<size_t>(4096 / ut);
  size_t f = ((static_cast<size_t>(Wa) * rt + 3) & ~size_t(3)) + 2 * kKC * static_cast<size_t>(ut);
  if (mode >= kRadFwd) f += rt * odd_stride(W2);
  if (mode == kRadDx) f += 8 * rt * odd_stride(W2);
  return f * sizeof(float);
}

template <int MODE, int UT>
__global__ void __launch_bounds__(256, UT == 64 ? 2 : 1) rowtile(RowtileArgs A) {
  constexpr bool RADIAL = MODE >= kRadFwd;
  constexpr bool DX = MODE == kUvuDx || MODE == kRadDx;
  constexpr int RT = rows_per_tile<UT>();
  constexpr int NUQ = UT / 4;  // channel quads per tile
  extern __shared__ __align__(16) float sm[];
  const UvuDev& t = A.t;
  const int W2a = odd_stride(A.W2);
  float* atile = sm;                                               // [Wa][RT]
  float* wtile = sm + ((static_cast<size_t>(A.Wa) * RT + 3) & ~size_t(3));  // [2][32 k][UT u]
  float* angt = wtile + 2 * kKC * UT;                              // [RT rows][W2a] (radial)
  float* dyp = angt + RT * W2a;                                    // [8 warps][RT][W2a] (kRadDx)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // a warp covers 4 channel quads x 8 row quads
  const int uq = (warp % (NUQ / 4)) * 4 + (lane & 3);
  const int rq = (warp / (NUQ / 4)) * 8 + (lane >> 2);
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * RT;
  const int ub = blockIdx.y * UT;
  const int u0 = ub + uq * 4;

  for (int idx = threadIdx.x; idx < RT * A.Wa; idx += blockDim.x) {
    const int c = idx % A.Wa, r = idx / A.Wa;
    const int64_t row = row0 + r;
    atile[c * RT + r] = row < A.rows ? __ldg(A.a_src + row * A.Wa + c) : 0.0f;
  }
  if (RADIAL) {
    for (int idx = threadIdx.x; idx < RT * A.W2; idx += blockDim.x) {
      const int c = idx % A.W2, r = idx / A.W2;
      const int64_t row = row0 + r;
      angt[r * W2a + c] = row < A.rows ? __ldg(A.ang + row * A.W2 + c) : 0.0f;
    }
    if (MODE == kRadDx)
      for (int idx = threadIdx.x; idx < 8 * RT * W2a; idx += blockDim.x) dyp[idx] = 0.f;
  }

  const int nkc = (A.K + kKC - 1) / kKC;
  const int ntiles = t.np * nkc;
  auto path_at = [&](int pos) { return DX ? t.by_i[pos] : pos; };
  auto issue = [&](int T, int buf) {
    const int p = path_at(T / nkc);
    const int k0 = (T % nkc) * kKC;
    float* dst = wtile + buf * (kKC * UT);
#pragma unroll
    for (int s = 0; s < kKC * NUQ / 256; ++s) {
      const int q = threadIdx.x + s * 256;  // float4 index in the tile
      const int kr = q / NUQ, c4 = q % NUQ;
      const int k = k0 + kr, u = ub + c4 * 4;
      const bool valid = k < A.K && u < A.Up;
      const float* src = valid ? A.wt + (static_cast<int64_t>(p) * A.K + k) * A.Up + u : A.wt;
      rt_cp_async16(dst + kr * UT + c4 * 4, src, valid);
    }
  };

  float acc[4][4][2];
  float proj[4][4][2];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[r][q][0] = acc[r][q][1] = proj[r][q][0] = proj[r][q][1] = 0.f;

  if (ntiles > 0) issue(0, 0);
  asm volatile("cp.async.commit_group;" ::: "memory");
  __syncthreads();
  for (int T = 0; T < ntiles; ++T) {
    if (T + 1 < ntiles) issue(T + 1, (T + 1) & 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    const int pos = T / nkc, kc = T % nkc;
    const int p = path_at(pos);
    const int4 pt = t.paths[p];  // (i, j, k)
    const int2 ej = t.in2[pt.y];
    const bool last_chunk = kc == nkc - 1;
    // operands of the coupling, loaded before the GEMM so that their latency hides
    float o[4][4][2], o2[4][4][2];
    const int2 eo = t.in1[DX ? pt.z : pt.x];
    const int2 eo2 = t.in1[pt.x];
    if (last_chunk) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t row = row0 + rq * 4 + r;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int u = u0 + q;
          const bool ok = row < A.rows && u < A.U;
          const float* s1 = A.opnd + row * A.W1 + eo.x + u * eo.y;
          o[r][q][0] = ok ? __ldg(s1) : 0.f;
          o[r][q][1] = (ok && eo.y == 2) ? __ldg(s1 + 1) : 0.f;
          if (MODE == kRadDx) {
            const float* s2 = A.opnd2 + row * A.W1 + eo2.x + u * eo2.y;
            o2[r][q][0] = ok ? __ldg(s2) : 0.f;
            o2[r][q][1] = (ok && eo2.y == 2) ? __ldg(s2 + 1) : 0.f;
          }
        }
      }
    }
    // GEMM over this k chunk
    const int db = RADIAL ? 1 : ej.y;
    const float* wb = wtile + (T & 1) * (kKC * UT) + uq * 4;
    const int kn = min(kKC, A.K - kc * kKC);
    auto step = [&](int kk, int nb) {
      const float4 w4 = *reinterpret_cast<const float4*>(wb + kk * UT);
      const int col = RADIAL ? kc * kKC + kk : ej.x + (kc * kKC + kk) * nb;
      const float4 y0 = *reinterpret_cast<const float4*>(atile + col * RT + rq * 4);
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
      const float ya[4] = {y0.x, y0.y, y0.z, y0.w};
      if (nb == 2) {
        const float4 y1 = *reinterpret_cast<const float4*>(atile + (col + 1) * RT + rq * 4);
        const float yb[4] = {y1.x, y1.y, y1.z, y1.w};
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            proj[r][q][0] = fmaf(ya[r], wv[q], proj[r][q][0]);
            proj[r][q][1] = fmaf(yb[r], wv[q], proj[r][q][1]);
          }
      } else {
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int q = 0; q < 4; ++q) proj[r][q][0] = fmaf(ya[r], wv[q], proj[r][q][0]);
      }
    };
    if (db == 2) {
      if (kn == kKC) {
#pragma unroll 4
        for (int kk = 0; kk < kKC; ++kk) step(kk, 2);
      } else {
        for (int kk = 0; kk < kn; ++kk) step(kk, 2);
      }
    } else {
      if (kn == kKC) {
#pragma unroll 4
        for (int kk = 0; kk < kKC; ++kk) step(kk, 1);
      } else {
        for (int kk = 0; kk < kn; ++kk) step(kk, 1);
      }
    }
    if (last_chunk) {
      float c[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) c[e] = __ldg(t.coef + 8 * p + e);
      float dyr[4][2];
#pragma unroll
      for (int r = 0; r < 4; ++r) dyr[r][0] = dyr[r][1] = 0.f;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float p0 = proj[r][q][0], p1 = proj[r][q][1];
          float wgt = 0.f;
          if (RADIAL) {
            const int u = u0 + q;
            wgt = p0 + ((A.bias != nullptr && u < A.U) ? __ldg(A.bias + p * A.U + u) : 0.f);
            const float* ay = angt + (rq * 4 + r) * W2a + ej.x;
            p0 = wgt * ay[0];
            p1 = ej.y == 2 ? wgt * ay[1] : 0.f;
          }
          const float o0 = o[r][q][0], o1 = o[r][q][1];
          if (!DX) {  // out[kc] += c[kc][a][b] x[a] q[b]
            acc[r][q][0] += c[0] * o0 * p0 + c[1] * o0 * p1 + c[2] * o1 * p0 + c[3] * o1 * p1;
            acc[r][q][1] += c[4] * o0 * p0 + c[5] * o0 * p1 + c[6] * o1 * p0 + c[7] * o1 * p1;
          } else {  // dx[a] += c[kc][a][b] g[kc] q[b]
            acc[r][q][0] += c[0] * o0 * p0 + c[1] * o0 * p1 + c[4] * o1 * p0 + c[5] * o1 * p1;
            acc[r][q][1] += c[2] * o0 * p0 + c[3] * o0 * p1 + c[6] * o1 * p0 + c[7] * o1 * p1;
          }
          if (MODE == kRadDx) {  // dy[b] += c[kc][a][b] g[kc] x[a] w
            const float x0 = o2[r][q][0], x1 = o2[r][q][1];
            dyr[r][0] += wgt * (c[0] * o0 * x0 + c[2] * o0 * x1 + c[4] * o1 * x0 + c[6] * o1 * x1);
            dyr[r][1] += wgt * (c[1] * o0 * x0 + c[3] * o0 * x1 + c[5] * o1 * x0 + c[7] * o1 * x1);
          }
          proj[r][q][0] = proj[r][q][1] = 0.f;
        }
      }
      if (MODE == kRadDx) {
        // reduce over the four u-quads of this warp (lanes differing in bits 0-1),
        // then one lane per row quad adds the warp's share (fixed order per warp)
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            float v = dyr[r][b];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            dyr[r][b] = v;
          }
        if ((lane & 3) == 0) {
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            float* d = dyp + (warp * RT + rq * 4 + r) * W2a + ej.x;
            d[0] += dyr[r][0];
            if (ej.y == 2) d[1] += dyr[r][1];
          }
        }
      }
      const int key = DX ? pt.x : pt.z;
      const bool last =
          pos + 1 == t.np ||
          (DX ? t.paths[path_at(pos + 1)].x : t.paths[path_at(pos + 1)].z) != key;
      if (last) {
        const int2 ek = t.in1[key];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int64_t row = row0 + rq * 4 + r;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int u = u0 + q;
            if (row < A.rows && u < A.U) {
              float* dst = A.out + row * A.W1 + ek.x + u * ek.y;
              dst[0] = acc[r][q][0];
              if (ek.y == 2) dst[1] = acc[r][q][1];
            }
            acc[r][q][0] = acc[r][q][1] = 0.f;
          }
        }
      }
    }
    __syncthreads();  // buffer T & 1 is refilled at T + 2
  }
  if (MODE == kRadDx) {
    // dy of the tile's rows: sum of the eight warps' shares in warp order
    for (int idx = threadIdx.x; idx < RT * A.W2; idx += blockDim.x) {
      const int r = idx / A.W2, col = idx % A.W2;
      const int64_t row = row0 + r;
      float s = 0.f;
      for (int w = 0; w < 8; ++w) s += dyp[(w * RT + r) * W2a + col];
      if (row < A.rows) A.dy[row * A.W2 + col] = s;
    }
  }
}

// Launches rowtile<MODE> with the 64-channel tile when the product has at most 64
// channels (no idle half tile), else the 128-channel tile.
template <int MODE>
int launch_rowtile(const RowtileArgs& ra, cudaStream_t stream) {
  const int ut = ra.U <= 64 ? 64 : kUT;
  const size_t smem = rowtile_smem(MODE, ut, ra.Wa, ra.W2);
  if (smem > 220 * 1024)
    return fail(ICTC_ERR_UNSUPPORTED, "operand rows too wide for the row tile (%zu bytes)", smem);
  const void* fn = ut == 64 ? reinterpret_cast<const void*>(&rowtile<MODE, 64>)
                            : reinterpret_cast<const void*>(&rowtile<MODE, kUT>);
  const int st = allow_smem(fn, smem);
  if (st != ICTC_OK) return st;
  const dim3 grid(static_cast<unsigned>(ceil_div(ra.rows, 4096 / ut)),
                  static_cast<unsigned>(ceil_div(ra.U, ut)));
  if (ut == 64)
    rowtile<MODE, 64><<<grid, 256, smem, stream>>>(ra);
  else
    rowtile<MODE, kUT><<<grid, 256, smem, stream>>>(ra);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "row tile launch");
}

}  // namespace ictc
