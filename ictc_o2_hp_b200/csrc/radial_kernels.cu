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

#include <cmath>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "rowtile.cuh"
#include "sgemm.cuh"
#include "tma.cuh"
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
// alpha [P * U, H] -> at [P][nt][H][TW]: channel tiles of width TW, zero past U.
// nt = 1, TW = Up is the plain [P][H][Up] layout of the row tile; the edge tile
// takes TW = its channel tile so each weight chunk is one contiguous copy.
__global__ void transpose_alpha(const float* __restrict__ a, float* __restrict__ at, int P, int U,
                                int TW, int nt, int H) {
  const int64_t total = static_cast<int64_t>(P) * nt * H * TW;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % TW);
    const int64_t rest = idx / TW;
    const int h = static_cast<int>(rest % H);
    const int64_t pt = rest / H;
    const int u = static_cast<int>(pt % nt) * TW + c;
    const int64_t p = pt / nt;
    at[idx] = u < U ? a[(p * U + u) * H + h] : 0.0f;
  }
}

// Channel tile of the edge tile kernel and the transposed-alpha width it needs.
inline int radial_ut(int U) { return U <= 64 ? 64 : 128; }
inline int radial_tiles(int U) { return (U + radial_ut(U) - 1) / radial_ut(U); }
inline size_t radial_at_bytes(int64_t P, int U, int H) {
  return static_cast<size_t>(P) * H * radial_tiles(U) * radial_ut(U) * sizeof(float);
}

// ------------------------------------------------------------ edge-weight gradient
//
// gw[e,p,u] = sum_{kc,a,b} c_p[kc][a][b] g_k[e,u,kc] x_i[e,u,a] y_j[e,b], the
// gradient of the regenerated edge weight w[e,p,u], is never stored: the dhidden
// and dalpha kernels rebuild it tile by tile from g, x and y.  Per edge the
// second input is folded into the coefficients first, C[kc][a] = sum_b c y_b,
// so gw = sum_{kc,a} C[kc][a] g[kc] x[a].  One thread builds eight consecutive
// channels of one edge; D1 and D3 (the dims of entries i and k) are compile-time
// so the operands stay in registers.

struct GwRegs {
  float x[16], g[16], y0, y1;
};

template <int D1, int D3>
__device__ __forceinline__ void gw8_load(GwRegs& r, const float* __restrict__ xrow,
                                         const float* __restrict__ grow,
                                         const float* __restrict__ yrow, int u0, int U, int2 ei,
                                         int2 ek, int2 ej, bool valid, bool vec) {
  const int nu = valid ? (U - u0 < 8 ? U - u0 : 8) : 0;
  const float* xs = xrow + ei.x + u0 * D1;
  const float* gs = grow + ek.x + u0 * D3;
  if (vec && nu == 8) {
#pragma unroll
    for (int q = 0; q < 2 * D1; ++q) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(xs) + q);
      r.x[4 * q] = v.x; r.x[4 * q + 1] = v.y; r.x[4 * q + 2] = v.z; r.x[4 * q + 3] = v.w;
    }
#pragma unroll
    for (int q = 0; q < 2 * D3; ++q) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(gs) + q);
      r.g[4 * q] = v.x; r.g[4 * q + 1] = v.y; r.g[4 * q + 2] = v.z; r.g[4 * q + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < 8 * D1; ++q) r.x[q] = q / D1 < nu ? __ldg(xs + q) : 0.f;
#pragma unroll
    for (int q = 0; q < 8 * D3; ++q) r.g[q] = q / D3 < nu ? __ldg(gs + q) : 0.f;
  }
  r.y0 = valid ? __ldg(yrow + ej.x) : 0.f;
  r.y1 = (valid && ej.y == 2) ? __ldg(yrow + ej.x + 1) : 0.f;
}

template <int D1, int D3>
__device__ __forceinline__ void gw8_compute(const GwRegs& r, const float (&c)[8],
                                            float (&out)[8]) {
  // C[kc][a] = c[kc][a][0] y0 + c[kc][a][1] y1 (coefficients at 4 kc + 2 a + b)
  const float c00 = fmaf(c[0], r.y0, c[1] * r.y1), c01 = fmaf(c[2], r.y0, c[3] * r.y1);
  const float c10 = fmaf(c[4], r.y0, c[5] * r.y1), c11 = fmaf(c[6], r.y0, c[7] * r.y1);
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const float x0 = r.x[u * D1], x1 = D1 == 2 ? r.x[u * D1 + 1] : 0.f;
    const float g0 = r.g[u * D3], g1 = D3 == 2 ? r.g[u * D3 + 1] : 0.f;
    float t0 = c00 * x0, t1 = 0.f;
    if (D1 == 2) t0 = fmaf(c01, x1, t0);
    if (D3 == 2) {
      t1 = c10 * x0;
      if (D1 == 2) t1 = fmaf(c11, x1, t1);
      out[u] = fmaf(g0, t0, g1 * t1);
    } else {
      out[u] = g0 * t0;
    }
  }
}

// Loads 4 channels x D values of one entry row segment (zeros past U).
template <int D>
__device__ __forceinline__ void ut_like_load(float (&v)[4 * D], const float* __restrict__ src,
                                             int u, int U, bool vec) {
  if (vec && u + 3 < U) {
#pragma unroll
    for (int q = 0; q < D; ++q) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(src) + q);
      v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4 * D; ++q) v[q] = u + q / D < U ? __ldg(src + q) : 0.f;
  }
}

// Runs body.template operator()<D1, D3>() for the entry dims of one path.
template <class Body>
__device__ __forceinline__ void with_dims(int d1, int d3, Body&& body) {
  if (d1 == 2) {
    if (d3 == 2) body.template operator()<2, 2>(); else body.template operator()<2, 1>();
  } else {
    if (d3 == 2) body.template operator()<1, 2>(); else body.template operator()<1, 1>();
  }
}

__device__ __forceinline__ void load_coef(const UvuDev& t, int p, float (&c)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) c[e] = __ldg(t.coef + 8 * p + e);
}

// 4 x 8 thread tile of a 64 x 64 CTA tile from k-major shared operands:
// rows m0..m0+3 of A[k][64], columns n0..n0+3 and n0+32..n0+35 of B[k][64].
template <int KS>
__device__ __forceinline__ void mma_4x8(const float (*A)[64], const float (*B)[64], int m0,
                                        int n0, float2 (&acc)[4][4]) {
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    const float4 a4 = *reinterpret_cast<const float4*>(&A[k][m0]);
    const float4 b0 = *reinterpret_cast<const float4*>(&B[k][n0]);
    const float4 b1 = *reinterpret_cast<const float4*>(&B[k][n0 + 32]);
    const float av[4] = {a4.x, a4.y, a4.z, a4.w};
    const float2 bv[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w),
                          make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fma2(av[i], bv[j], acc[i][j]);
  }
}

// ------------------------------------------------------------ forward and dx / dy
//
// radial_tile<MODE, UT>: a CTA owns RT edges x UT channels and walks the paths.
// Per path p it regenerates the edge weights of its tile,
//   w[e,p,u] = sum_h hidden[e,h] alpha[p*U+u, h] (+ bias),
// as a GEMM (K = H in chunks of 64; the hidden tile stays in shared memory for
// the whole CTA, alpha_p streams through a cp.async double buffer), with 256
// threads in 4 edge x 8 channel tiles (channels tc*4..+3 and UT/2 + tc*4..+3).
// The coupling then folds the second input into the coefficients per edge,
// C[kc][a] = sum_b c_p[kc][a][b] y_j[e,b], and
//   forward:  out_k[e,u,kc] += w sum_a C[kc][a] x_i[e,u,a]   (paths grouped by k)
//   dx mode:  dx_i[e,u,a]   += w sum_kc C[kc][a] g_k[e,u,kc]  (paths grouped by i)
//             dy_j[e,b]     += sum_u w sum_{kc,a} c[kc][a][b] g_k x_i
// The accumulators of the current k (or i) group stay in registers; dy is
// reduced over the tile's channels with shuffles, then added per path in path
// order into a shared per-edge row (deterministic).  Path metadata is copied to
// shared memory once per CTA.
enum RadTileMode { kRtFwd = 0, kRtDx = 1 };
constexpr int kRtThreads = 256;
constexpr int kRtKC = 64;     // hidden features per weight chunk
constexpr int kRtStages = 4;  // weight chunks in flight

struct RadTileArgs {
  const float* opnd;    // forward: x; dx mode: g   [rows, W1]
  const float* x;       // dx mode: x               [rows, W1]
  const float* hidden;  // [rows, H]
  const float* ang;     // [rows, W2]
  const float* at;      // alpha as [P][H][Up]
  const float* bias;    // [P * U] or null
  float* out;           // forward output or dx     [rows, W1]
  float* dy;            // dx mode                  [rows, W2]
  int64_t rows;
  int U, Up, H, W1, W2;
  UvuDev t;
  bool vec;  // 16-byte access to 4-channel groups of opnd / x / out
  float* gw = nullptr;  // dx mode, optional: edge-weight gradient [rows][Wn]
  int64_t Wn = 0;
  // optional gather of the first input: row e of x is row xrow[e] of the x source
  // (forward: opnd, dx mode: x), which has xrows rows; null = row e itself
  const int64_t* xrow = nullptr;
  int64_t xrows = 0;
};

// Device error code of an x-row index outside [0, xrows) (the row reads as zeros).
constexpr int kBadGatherIndex = 17;

// Thread tiles: 4 edges x NH groups of 4 channels (NH = 2: 256 threads, the 4x8
// "split" tile; NH = 1: 512 threads, the 4x4 "wide" tile with half the registers
// per thread and twice the warps).  Both cover RT = 128 (UT = 64) or 64 (UT = 128)
// edges per CTA.
template <int UT, int NH = 2>
struct RtShape {
  static constexpr int NC = NH == 2 ? 2 : 1;                  // channel groups per thread
  static constexpr int NT = NH == 2 ? 256 : (NH == 1 ? 512 : 384);  // threads per CTA
  static constexpr int TC = UT / (4 * NC);                    // threads along the channels
  static constexpr int TR = NT / TC;                          // thread rows
  static constexpr int RT = TR * 4;                           // edges per CTA
};

inline size_t radial_tile_smem(int ut, int H, int W2, int np, int n1, int n2, bool dx,
                               int rt_edges = 0) {
  const size_t rt = rt_edges > 0 ? static_cast<size_t>(rt_edges)
                                 : static_cast<size_t>(kRtThreads / (ut / 8)) * 4;
  const size_t kc = static_cast<size_t>(H < kRtKC ? H : kRtKC);
  const size_t w2s = static_cast<size_t>(odd_stride(W2));
  const size_t floats = static_cast<size_t>(H) * rt + kRtStages * kc * ut + rt * w2s +
                        static_cast<size_t>(np) * 8 + (dx ? rt * w2s : 0);
  const size_t aligned_floats = (floats + 3) & ~size_t(3);
  const size_t ints = static_cast<size_t>(np) * 4 + static_cast<size_t>(n1 + n2) * 2 + np;
  const size_t rows64 = rt;  // x row of each edge of the tile
  return 128 + (aligned_floats + ints) * 4 + 8 + rows64 * 8;
}

// Loads 4 channels x D values of one entry of one row (zeros past U or rows).
template <int D>
__device__ __forceinline__ void load4(float (&v)[4 * D], const float* __restrict__ src,
                                      bool row_ok, int u, int U, bool vec) {
  if (vec && row_ok && u + 3 < U) {
#pragma unroll
    for (int q = 0; q < D; ++q) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(src) + q);
      v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4 * D; ++q) v[q] = (row_ok && u + q / D < U) ? __ldg(src + q) : 0.f;
  }
}

template <int D>
__device__ __forceinline__ void store4(float* __restrict__ dst, const float (&v)[4][2],
                                       bool row_ok, int u, int U, bool vec) {
  if (!row_ok) return;
  if (vec && u + 3 < U) {
#pragma unroll
    for (int q = 0; q < D; ++q) {
      float4 t;
      t.x = v[(4 * q) / D][(4 * q) % D];
      t.y = v[(4 * q + 1) / D][(4 * q + 1) % D];
      t.z = v[(4 * q + 2) / D][(4 * q + 2) % D];
      t.w = v[(4 * q + 3) / D][(4 * q + 3) % D];
      reinterpret_cast<float4*>(dst)[q] = t;
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4 * D; ++q)
      if (u + q / D < U) dst[q] = v[q / D][q % D];
  }
}

// GX: the first input is gathered (row e of x is row A.xrow[e] of the source); the
// kernel is compiled without the per-edge row lookups when it is not.
template <int MODE, int UT, int NH, bool GX>
__global__ void __launch_bounds__(RtShape<UT, NH>::NT, 1) radial_tile(RadTileArgs A) {
  using Sh = RtShape<UT, NH>;
  constexpr int RT = Sh::RT, TC = Sh::TC, NT = Sh::NT, NC = Sh::NC;
  constexpr int CW = 4 * NC;  // channels per thread
  extern __shared__ __align__(128) unsigned char rt_raw[];
  // [0, 128): stage barriers (full) and release counters
  uint64_t* full = reinterpret_cast<uint64_t*>(rt_raw);
  unsigned* done = reinterpret_cast<unsigned*>(rt_raw + 64);
  float* sm = reinterpret_cast<float*>(rt_raw + 128);
  const int tid = threadIdx.x, lane = tid & 31;
  const int nwarps = NT / 32;
  const int kc = A.H < kRtKC ? A.H : kRtKC;
  const int nkc = (A.H + kRtKC - 1) / kRtKC;
  const int W2s = odd_stride(A.W2);
  const int np = A.t.np;
  float* Ht = sm;                                          // [H][RT]
  float* Wt = Ht + static_cast<size_t>(A.H) * RT;          // [kRtStages][kc][UT]
  float* angt = Wt + kRtStages * kc * UT;                  // [RT][W2s]
  float* coef = angt + RT * W2s;                           // [np][8]
  float* dyacc = coef + np * 8;                            // [RT][W2s] (dx mode)
  float* fend = dyacc + (MODE == kRtDx ? RT * W2s : 0);
  int4* paths = reinterpret_cast<int4*>(sm + ((fend - sm + 3) & ~3));
  int2* in1 = reinterpret_cast<int2*>(paths + np);
  int2* in2 = in1 + A.t.n1;
  int* order = reinterpret_cast<int*>(in2 + A.t.n2);
  // x source row of each edge of the tile (-1: past the rows or a bad index)
  int64_t* xr = reinterpret_cast<int64_t*>(
      (reinterpret_cast<uintptr_t>(order + np) + 7) & ~static_cast<uintptr_t>(7));
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * RT;
  // Channel tiles: the forward spreads them over blockIdx.y; the dx mode walks them
  // inside the CTA (dy sums over every channel, so one CTA owns an edge's dy).
  const int nub = MODE == kRtDx ? (A.U + UT - 1) / UT : 1;
  auto tile_ub = [&](int T) {
    return MODE == kRtDx ? (T / (np * nkc)) * UT : static_cast<int>(blockIdx.y) * UT;
  };

  for (int q = tid; q < np; q += NT) {
    paths[q] = A.t.paths[q];
    order[q] = MODE == kRtDx ? A.t.by_i[q] : q;
  }
  for (int q = tid; q < np * 8; q += NT) coef[q] = __ldg(A.t.coef + q);
  for (int q = tid; q < A.t.n1; q += NT) in1[q] = A.t.in1[q];
  for (int q = tid; q < A.t.n2; q += NT) in2[q] = A.t.in2[q];
  if constexpr (GX) {
    for (int r = tid; r < RT; r += NT) {
      const int64_t row = row0 + r;
      int64_t v = -1;
      if (row < A.rows) {
        v = __ldg(A.xrow + row);
        if (v < 0 || v >= A.xrows) {
          atomicExch(&g_ictc_device_error, kBadGatherIndex);
          v = -1;
        }
      }
      xr[r] = v;
    }
  }
  for (int idx = tid; idx < RT * A.H; idx += NT) {
    const int r = idx / A.H, h = idx - r * A.H;
    const int64_t row = row0 + r;
    Ht[h * RT + r] = row < A.rows ? __ldg(A.hidden + row * A.H + h) : 0.f;
  }
  for (int idx = tid; idx < RT * A.W2; idx += NT) {
    const int r = idx / A.W2, c = idx - r * A.W2;
    const int64_t row = row0 + r;
    angt[r * W2s + c] = row < A.rows ? __ldg(A.ang + row * A.W2 + c) : 0.f;
  }
  if (MODE == kRtDx)
    for (int idx = tid; idx < RT * W2s; idx += NT) dyacc[idx] = 0.f;
  if (tid == 0) {
    for (int st = 0; st < kRtStages; ++st) {
      mbar_init(&full[st], 1);
      done[st] = 0;
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  const int tc = tid % TC, tr = tid / TC;
  const int e0 = tr * 4;
  const int ntiles = nub * np * nkc;
  // One thread copies weight chunk T (rows k0.. of alpha_p, channel tile ub / UT)
  // into stage st: alpha is laid out [P][channel tiles][H][UT] (zero past U), so a
  // chunk is one contiguous bulk asynchronous copy.
  const int ntl = (A.U + UT - 1) / UT;
  auto issue = [&](int T, int st) {
    const int p = order[(T / nkc) % np], k0 = (T % nkc) * kRtKC;
    const int kn = A.H - k0 < kRtKC ? A.H - k0 : kRtKC;
    float* dst = Wt + st * kc * UT;
    const float* src =
        A.at + ((static_cast<int64_t>(p) * ntl + tile_ub(T) / UT) * A.H + k0) * UT;
    const uint32_t bytes = static_cast<uint32_t>(kn) * UT * 4u;
    mbar_arrive_expect_tx(&full[st], bytes);
    bulk_g2s(dst, src, bytes, &full[st]);
  };

  float2 acc[4][CW / 2];  // edge-weight tile, paired along the channels
  float2 res[4][CW];  // output (forward) or dx (dx mode) components of each channel
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < CW; ++b) res[a][b] = make_float2(0.f, 0.f);

  if (tid == 0)
    for (int T = 0; T < kRtStages && T < ntiles; ++T) issue(T, T);
  bool ok = true;
  // (channel tile, path position, hidden chunk) of tile T, advanced per tile: T runs
  // over ck fastest, then pos, then the channel tile (no division per tile)
  int ck = 0, pos = 0, ub = tile_ub(0);
  auto advance = [&]() {
    if (++ck == nkc) {
      ck = 0;
      if (++pos == np) {
        pos = 0;
        ub += UT;
      }
    }
  };
  for (int T = 0; T < ntiles && ok; ++T, advance()) {
    const int st = T % kRtStages;
    const uint32_t round = static_cast<uint32_t>(T / kRtStages);
    ok = mbar_wait(&full[st], round & 1, 5);
    if (!ok) break;
    const int p = order[pos];
    if (ck == 0) {
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < CW / 2; ++b) acc[a][b] = make_float2(0.f, 0.f);
      // Pull the path's epilogue operands (x_i; g_k in dx mode) of this thread's
      // four edges toward L1 while the path's product runs: lane tc takes line tc
      // of each edge's slice, lines that start inside the valid channels only.
      const int4 pt = paths[p];
      const int2 ea = in1[pt.x], eb = in1[pt.z];
      const int uspan = A.U - ub < UT ? A.U - ub : UT;
#pragma unroll
      for (int ee = 0; ee < 4; ++ee) {
        const int64_t row = row0 + e0 + ee;
        const int64_t xrow = GX ? xr[e0 + ee] : row;
        if (row < A.rows) {
          if (xrow >= 0) {
            const float* xp = (MODE == kRtFwd ? A.opnd : A.x) + xrow * A.W1 + ea.x +
                              static_cast<int64_t>(ub) * ea.y;
            if (tc * 32 < uspan * ea.y) prefetch_l1(xp + tc * 32);
          }
          if (MODE == kRtDx) {
            const float* gr = A.opnd + row * A.W1 + eb.x + static_cast<int64_t>(ub) * eb.y;
            if (tc * 32 < uspan * eb.y) prefetch_l1(gr + tc * 32);
          }
        }
      }
    }
    const int kn = A.H - ck * kRtKC < kRtKC ? A.H - ck * kRtKC : kRtKC;
    const float* Wb = Wt + st * kc * UT;
    const float* Hb = Ht + static_cast<size_t>(ck) * kRtKC * RT;
    auto kstep = [&](int k) {
      const float4 a4 = *reinterpret_cast<const float4*>(Hb + k * RT + e0);
      const float av[4] = {a4.x, a4.y, a4.z, a4.w};
      float2 bv[CW / 2];
#pragma unroll
      for (int h = 0; h < NC; ++h) {
        const float4 b4 = *reinterpret_cast<const float4*>(Wb + k * UT + h * (UT / NC) + tc * 4);
        bv[2 * h] = make_float2(b4.x, b4.y);
        bv[2 * h + 1] = make_float2(b4.z, b4.w);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < CW / 2; ++j) acc[i][j] = fma2(av[i], bv[j], acc[i][j]);
    };
    if (kn == kRtKC) {
      // the forward and the 512-thread dx tile unroll a full chunk completely; the
      // 384-thread dx tile by 8 (fully unrolled it was 4 % slower at config 5)
      if constexpr (MODE == kRtFwd || NH == 1) {
#pragma unroll
        for (int k = 0; k < kRtKC; ++k) kstep(k);
      } else {
#pragma unroll 8
        for (int k = 0; k < kRtKC; ++k) kstep(k);
      }
    } else {
      for (int k = 0; k < kn; ++k) kstep(k);
    }
    // release the stage; the last warp out refills it (no warp waits here)
    __syncwarp();
    if (lane == 0) {
      unsigned prev;
      asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                   : "=r"(prev)
                   : "r"(smem_addr(&done[st]))
                   : "memory");
      if (prev + 1 == static_cast<unsigned>(nwarps) * (round + 1)) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (T + kRtStages < ntiles) issue(T + kRtStages, st);
      }
    }
    if (ck == nkc - 1) {
      const int4 pt = paths[p];
      const int2 ei = in1[pt.x], ej = in2[pt.y], ek = in1[pt.z];
      const float* c = coef + 8 * p;
      const int key = MODE == kRtFwd ? pt.z : pt.x;
      // The coefficient pairs below feed paired f32x2 operations (`fma2`, `__fmul2_rn`):
      // each component is computed in the same operation order as the scalar form,
      // so the results are bit-identical to it with half the issue slots.
      const float2 k01 = make_float2(c[0], c[1]), k23 = make_float2(c[2], c[3]);
      const float2 k45 = make_float2(c[4], c[5]), k67 = make_float2(c[6], c[7]);
      with_dims(ei.y, ek.y, [&]<int D1, int D3>() {
#pragma unroll
        for (int ee = 0; ee < 4; ++ee) {
          const int r = e0 + ee;
          const int64_t row = row0 + r;
          const bool row_ok = row < A.rows;
          const int64_t xrw = GX ? xr[r] : (row_ok ? row : -1);  // x source row (-1: none)
          const bool x_ok = xrw >= 0;
          const int64_t xoff = (x_ok ? xrw : 0) * A.W1;
          const float y0 = angt[r * W2s + ej.x];
          const float y1 = ej.y == 2 ? angt[r * W2s + ej.x + 1] : 0.f;
          // C[kc][a] = sum_b c[4 kc + 2 a + b] y_b
          const float c00 = fmaf(c[0], y0, c[1] * y1), c01 = fmaf(c[2], y0, c[3] * y1);
          const float c10 = fmaf(c[4], y0, c[5] * y1), c11 = fmaf(c[6], y0, c[7] * y1);
          float2 dyp = make_float2(0.f, 0.f);
#pragma unroll
          for (int half = 0; half < NC; ++half) {
            const int u = ub + half * (UT / NC) + tc * 4;
            if (MODE == kRtFwd) {
              float xv[4 * D1];
              load4<D1>(xv, A.opnd + xoff + ei.x + static_cast<int64_t>(u) * D1, x_ok, u, A.U,
                        A.vec);
              // out[kc] += w sum_a C[kc][a] x[a], both kc at once: (C00, C10) x0 + (C01, C11) x1
              const float2 ca0 = make_float2(c00, c10), ca1 = make_float2(c01, c11);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float w = pair_at(acc[ee], half * 4 + q);
                if (A.bias != nullptr && u + q < A.U) w += __ldg(A.bias + p * A.U + u + q);
                const float x0 = xv[q * D1], x1 = D1 == 2 ? xv[q * D1 + 1] : 0.f;
                float2& o = res[ee][half * 4 + q];
                if (D3 == 2) {
                  float2 t = __fmul2_rn(make_float2(x0, x0), ca0);
                  if (D1 == 2) t = fma2(x1, ca1, t);
                  o = fma2(w, t, o);
                } else {
                  float t0 = c00 * x0;
                  if (D1 == 2) t0 = fmaf(c01, x1, t0);
                  o.x = fmaf(w, t0, o.x);
                }
              }
            } else {
              float gv[4 * D3], xv[4 * D1];
              load4<D3>(gv, A.opnd + row * A.W1 + ek.x + static_cast<int64_t>(u) * D3, row_ok, u,
                        A.U, A.vec);
              load4<D1>(xv, A.x + xoff + ei.x + static_cast<int64_t>(u) * D1, x_ok, u, A.U,
                        A.vec);
              // dx[a] += w sum_kc C[kc][a] g[kc], both a at once: (C00, C01) g0 + (C10, C11) g1
              const float2 ck0 = make_float2(c00, c01), ck1 = make_float2(c10, c11);
              float gwv[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float w = pair_at(acc[ee], half * 4 + q);
                if (A.bias != nullptr && u + q < A.U) w += __ldg(A.bias + p * A.U + u + q);
                const float g0 = gv[q * D3], g1 = D3 == 2 ? gv[q * D3 + 1] : 0.f;
                const float x0 = xv[q * D1], x1 = D1 == 2 ? xv[q * D1 + 1] : 0.f;
                float2& o = res[ee][half * 4 + q];
                if (D1 == 2) {
                  float2 sv = __fmul2_rn(ck0, make_float2(g0, g0));
                  if (D3 == 2) sv = fma2(g1, ck1, sv);
                  o = fma2(w, sv, o);
                } else {
                  float s0 = c00 * g0;
                  if (D3 == 2) s0 = fmaf(c10, g1, s0);
                  o.x = fmaf(w, s0, o.x);
                }
                // (dy0, dy1) += w sum_{kc,a} (c[4 kc + 2 a], c[4 kc + 2 a + 1]) g[kc] x[a]
                float2 d = __fmul2_rn(__fmul2_rn(k01, make_float2(g0, g0)), make_float2(x0, x0));
                if (D1 == 2) d = fma2(x1, __fmul2_rn(k23, make_float2(g0, g0)), d);
                if (D3 == 2) d = fma2(x0, __fmul2_rn(k45, make_float2(g1, g1)), d);
                if (D1 == 2 && D3 == 2) d = fma2(x1, __fmul2_rn(k67, make_float2(g1, g1)), d);
                dyp = fma2(w, d, dyp);
                // gw = sum_b y_b sum_{kc,a} c[kc][a][b] g[kc] x[a]
                gwv[q] = fmaf(y0, d.x, y1 * d.y);
              }
              if (A.gw != nullptr && row_ok) {
                // streaming stores (evict first): the gw block is far larger than L2
                // and would otherwise push out the x rows the later paths re-read
                float* dst = A.gw + row * A.Wn + static_cast<int64_t>(p) * A.U + u;
                if (A.vec && u + 3 < A.U) {
                  __stcs(reinterpret_cast<float4*>(dst), make_float4(gwv[0], gwv[1], gwv[2], gwv[3]));
                } else {
#pragma unroll
                  for (int q = 0; q < 4; ++q)
                    if (u + q < A.U) __stcs(dst + q, gwv[q]);
                }
              }
            }
          }
          if (MODE == kRtDx) {
            // sum over the TC threads that share these edges (consecutive lanes)
            float dyp0 = dyp.x, dyp1 = dyp.y;
#pragma unroll
            for (int m = 1; m < TC; m <<= 1) {
              dyp0 += __shfl_xor_sync(0xffffffffu, dyp0, m);
              dyp1 += __shfl_xor_sync(0xffffffffu, dyp1, m);
            }
            if (tc == 0) {
              dyacc[r * W2s + ej.x] += dyp0;
              if (ej.y == 2) dyacc[r * W2s + ej.x + 1] += dyp1;
            }
          }
        }
      });
      const bool last = pos + 1 == np ||
                        (MODE == kRtFwd ? paths[order[pos + 1]].z : paths[order[pos + 1]].x) != key;
      if (last) {
        const int2 eo = in1[key];
        const int dd = eo.y;
#pragma unroll
        for (int ee = 0; ee < 4; ++ee) {
          const int64_t row = row0 + e0 + ee;
          const bool row_ok = row < A.rows;
#pragma unroll
          for (int half = 0; half < NC; ++half) {
            const int u = ub + half * (UT / NC) + tc * 4;
            float v[4][2];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              v[q][0] = res[ee][half * 4 + q].x;
              v[q][1] = res[ee][half * 4 + q].y;
            }
            float* dst = A.out + row * A.W1 + eo.x + static_cast<int64_t>(u) * dd;
            if (dd == 2) store4<2>(dst, v, row_ok, u, A.U, A.vec);
            else store4<1>(dst, v, row_ok, u, A.U, A.vec);
          }
#pragma unroll
          for (int b = 0; b < CW; ++b) res[ee][b] = make_float2(0.f, 0.f);
        }
      }
    }
  }
  if (!ok && tid == 0) {
    // a wait ran out: let copies already issued land before the CTA exits
    for (int st = 0; st < kRtStages; ++st) mbar_wait(&full[st], 0, 6, kDrainLimitNs);
  }
  if (MODE == kRtDx) {
    __syncthreads();
    for (int idx = tid; idx < RT * A.W2; idx += NT) {
      const int r = idx / A.W2, col = idx - r * A.W2;
      const int64_t row = row0 + r;
      if (row < A.rows) A.dy[row * A.W2 + col] = dyacc[r * W2s + col];
    }
  }
}

// Whether the edge tile's shared memory (resident hidden tile, weight ring, path
// metadata) fits; otherwise the row tile runs, on the [P][H][Up] alpha layout.
inline bool radial_tile_fits(int U, int H, int W2, int np, int n1, int n2, bool dx) {
  return radial_tile_smem(radial_ut(U), H, W2, np, n1, n2, dx) <= 225 * 1024;
}

template <int MODE, int UT, int NH, bool GX>
int launch_radial_tile_gx(const RadTileArgs& ra, size_t smem, cudaStream_t s) {
  using Sh = RtShape<UT, NH>;
  const void* fn = reinterpret_cast<const void*>(&radial_tile<MODE, UT, NH, GX>);
  const int st = allow_smem(fn, smem);
  if (st != ICTC_OK) return st;
  const dim3 grid(static_cast<unsigned>(ceil_div(ra.rows, Sh::RT)),
                  MODE == kRtDx ? 1u : static_cast<unsigned>(ceil_div(ra.U, UT)));
  radial_tile<MODE, UT, NH, GX><<<grid, Sh::NT, smem, s>>>(ra);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "radial tile launch");
}

template <int MODE, int UT, int NH>
int launch_radial_tile_shape(const RadTileArgs& ra, size_t smem, cudaStream_t s) {
  return ra.xrow != nullptr ? launch_radial_tile_gx<MODE, UT, NH, true>(ra, smem, s)
                            : launch_radial_tile_gx<MODE, UT, NH, false>(ra, smem, s);
}

// Thread tile of the edge tile kernel, all 4 edges x 4 channels per thread except
// "split": "wide" = 512 threads (128 registers, 16 warps per SM: the forward's shape),
// "mid" = 384 threads (up to 170 registers, 12 warps per SM), "split" = 4 x 8 on 256
// threads.  Both wide and mid run one CTA per SM.  At 512 threads the dx tile spills;
// the mid tile took it 32.7 -> 31.0 ms at config 5 (1,048,576 edges), but its smaller
// edge tile leaves a fuller last wave at some sizes (C64 m6 at 131,072 edges: 9.2 waves
// of mid CTAs, 13.9 vs 14.3 ms for wide), so the dx tile takes mid when its speed
// (about 5 %) outweighs the difference in last-wave fill.  ICTC_RADIAL_TILE=
// wide|mid|split forces one shape for both modes (tests cover each).
enum RtTile { kTileWide = 1, kTileSplit = 2, kTileMid = 3 };

template <int UT>
inline int radial_tile_shape(int mode, int64_t rows) {
  const char* v = getenv("ICTC_RADIAL_TILE");
  if (v != nullptr) {
    if (strcmp(v, "split") == 0) return kTileSplit;
    if (strcmp(v, "mid") == 0) return kTileMid;
    if (strcmp(v, "wide") == 0) return kTileWide;
  }
  if (mode != kRtDx) return kTileWide;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return kTileWide;
  const double sms = sm_count(device);
  auto fill = [&](int rt) {  // busy fraction of the SM-waves the launch occupies
    const double ctas = static_cast<double>((rows + rt - 1) / rt);
    return ctas / (sms * std::ceil(ctas / sms));
  };
  return fill(RtShape<UT, 3>::RT) * 1.05 >= fill(RtShape<UT, 1>::RT) ? kTileMid : kTileWide;
}

template <int MODE, int UT>
int launch_radial_tile_ut(const RadTileArgs& ra, cudaStream_t s) {
  auto smem = [&](int rt) {
    return radial_tile_smem(UT, ra.H, ra.W2, ra.t.np, ra.t.n1, ra.t.n2, MODE == kRtDx, rt);
  };
  switch (radial_tile_shape<UT>(MODE, ra.rows)) {
    case kTileSplit:
      return launch_radial_tile_shape<MODE, UT, 2>(ra, smem(RtShape<UT, 2>::RT), s);
    case kTileMid:
      return launch_radial_tile_shape<MODE, UT, 3>(ra, smem(RtShape<UT, 3>::RT), s);
    default:
      return launch_radial_tile_shape<MODE, UT, 1>(ra, smem(RtShape<UT, 1>::RT), s);
  }
}

template <int MODE>
int launch_radial_tile(const RadTileArgs& ra, cudaStream_t s) {
  const int ut = radial_ut(ra.U);
  const size_t smem = radial_tile_smem(ut, ra.H, ra.W2, ra.t.np, ra.t.n1, ra.t.n2, MODE == kRtDx);
  if (smem > 225 * 1024) return ICTC_ERR_UNSUPPORTED;  // caller falls back to the row tile
  return ut == 64 ? launch_radial_tile_ut<MODE, 64>(ra, s) : launch_radial_tile_ut<MODE, 128>(ra, s);
}

// ------------------------------------------------------------ dhidden
//
// dh[e,h] = sum_{p,u} gw[e,p,u] alpha[p*U+u, h]: a GEMM over K = (p, u) in steps of
// 16 channels.  CTA of 128 threads for a 64 edge x 64 h tile (thread tile 4 edges x
// 8 h).  Per step the gw tile [16 u][64 e] is built from g, x, y and the alpha rows
// [16 u][64 h] are copied into shared memory; both double-buffered, the next
// step's operands fetched into registers before this step's GEMM.
constexpr int kDhE = 64, kDhH = 64, kDhU = 16;

struct DhArgs {
  const float* x; const float* ang; const float* g; const float* alpha; float* dh;
  int64_t rows; int U, H, W1, W2; UvuDev t; bool vec, avec;
};

__global__ void __launch_bounds__(128, 4) radial_dhidden(DhArgs A) {
  __shared__ __align__(16) float gwt[2][kDhU][kDhE];
  __shared__ __align__(16) float at[2][kDhU][kDhH];
  const int tid = threadIdx.x;
  const int64_t e_base = static_cast<int64_t>(blockIdx.x) * kDhE;
  const int hb = blockIdx.y * kDhH;
  // generation: edge ge (lanes = consecutive edges), channel octet go (warp-uniform)
  const int ge = tid & 63, go = tid >> 6;
  const int64_t grow_i = e_base + ge;
  const bool gvalid = grow_i < A.rows;
  const float* xrow = A.x + (gvalid ? grow_i : 0) * A.W1;
  const float* gr = A.g + (gvalid ? grow_i : 0) * A.W1;
  const float* yrow = A.ang + (gvalid ? grow_i : 0) * A.W2;
  // GEMM: edges m0..m0+3, h n0..n0+3 and n0+32..n0+35
  const int m0 = (tid >> 3) * 4, n0 = (tid & 7) * 4;
  const int nuc = (A.U + kDhU - 1) / kDhU;
  const int nsteps = A.t.np * nuc;
  float2 acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = make_float2(0.f, 0.f);

  GwRegs r;
  float4 av[2];
  int cur_d1 = 1, cur_d3 = 1;
  float c[8];
  auto fetch = [&](int step) {
    const int p = step / nuc, uc = step % nuc;
    const int4 pt = A.t.paths[p];
    const int2 ei = A.t.in1[pt.x], ej = A.t.in2[pt.y], ek = A.t.in1[pt.z];
    cur_d1 = ei.y;
    cur_d3 = ek.y;
    load_coef(A.t, p, c);
    const int u0 = uc * kDhU + go * 8;
    with_dims(ei.y, ek.y, [&]<int D1, int D3>() {
      gw8_load<D1, D3>(r, xrow, gr, yrow, u0, A.U, ei, ek, ej, gvalid && u0 < A.U, A.vec);
    });
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int q = tid + s * 128;
      const int uu = q >> 4, h = hb + (q & 15) * 4;
      const int u = uc * kDhU + uu;
      const float* src = A.alpha + (static_cast<int64_t>(p) * A.U + u) * A.H + h;
      if (u < A.U && A.avec && h + 3 < A.H) {
        av[s] = __ldg(reinterpret_cast<const float4*>(src));
      } else {
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = (u < A.U && h + k < A.H) ? __ldg(src + k) : 0.f;
        av[s] = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
  };
  auto stash = [&](int buf) {
    float out[8];
    with_dims(cur_d1, cur_d3, [&]<int D1, int D3>() { gw8_compute<D1, D3>(r, c, out); });
#pragma unroll
    for (int i = 0; i < 8; ++i) gwt[buf][go * 8 + i][ge] = out[i];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int q = tid + s * 128;
      *reinterpret_cast<float4*>(&at[buf][q >> 4][(q & 15) * 4]) = av[s];
    }
  };
  if (nsteps > 0) {
    fetch(0);
    stash(0);
  }
  __syncthreads();
  for (int step = 0; step < nsteps; ++step) {
    const int buf = step & 1;
    const bool more = step + 1 < nsteps;
    if (more) fetch(step + 1);
    mma_4x8<kDhU>(gwt[buf], at[buf], m0, n0, acc);
    if (more) stash(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t e = e_base + m0 + a;
    if (e >= A.rows) continue;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int h = hb + n0 + (b & 3) + (b >> 2) * 32;
      if (h < A.H) A.dh[e * A.H + h] = pair_at(acc[a], b);
    }
  }
}

// ------------------------------------------------------------ dalpha, dbias
//
// dalpha[p*U+u, h] = sum_e gw[e,p,u] hidden[e,h] and dbias[p*U+u] = sum_e gw[e,p,u]:
// per CTA (128 threads) one path, a 64 u x 64 h tile (thread tile 4 u x 8 h) and
// one chunk of the edges (partials are summed over chunks in a fixed order
// afterwards).  K = edges in steps of 16: the gw tile [16 e][64 u] is built on
// chip, the hidden rows [16 e][64 h] copied, both double-buffered with register
// prefetch of the next step.
constexpr int kDaE = 16, kDaU = 64, kDaH = 64;

struct DaArgs {
  const float* x; const float* ang; const float* g; const float* hidden;
  float* da; float* db; int64_t rows, chunk_rows, da_numel, db_numel;
  int U, H, W1, W2; UvuDev t; bool vec, hvec;
};

template <int D1, int D3>
__device__ __forceinline__ void radial_dalpha_body(const DaArgs& A, float (*gwt)[kDaE][kDaU],
                                                   float (*ht)[kDaE][kDaH], float* red) {
  const int tid = threadIdx.x;
  const int p = blockIdx.x;
  const int nut = (A.U + kDaU - 1) / kDaU;
  const int ub = (blockIdx.y % nut) * kDaU, hb = (blockIdx.y / nut) * kDaH;
  const int4 pt = A.t.paths[p];
  const int2 ei = A.t.in1[pt.x], ej = A.t.in2[pt.y], ek = A.t.in1[pt.z];
  float c[8];
  load_coef(A.t, p, c);
  // generation: edge ge of the step, channels ub + go*8 .. +7
  const int ge = tid >> 3, go = tid & 7;
  const int u0g = ub + go * 8;
  // GEMM: u m0..m0+3 (tile-relative), h n0..n0+3 and n0+32..n0+35
  const int m0 = (tid >> 3) * 4, n0 = (tid & 7) * 4;
  const int64_t rbeg = static_cast<int64_t>(blockIdx.z) * A.chunk_rows;
  const int64_t rend = rbeg + A.chunk_rows < A.rows ? rbeg + A.chunk_rows : A.rows;
  float2 acc[4][4];
  float bsum[8];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 8; ++i) bsum[i] = 0.f;
  GwRegs r;
  float4 hv[2];
  auto fetch = [&](int64_t e0) {
    const int64_t e = e0 + ge;
    const bool valid = e < rend && u0g < A.U;
    const int64_t row = e < rend ? e : rbeg;
    gw8_load<D1, D3>(r, A.x + row * A.W1, A.g + row * A.W1, A.ang + row * A.W2, u0g, A.U, ei,
                     ek, ej, valid, A.vec);
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int q = tid + s * 128;
      const int er = q >> 4, h = hb + (q & 15) * 4;
      const int64_t ee = e0 + er;
      const float* src = A.hidden + (ee < rend ? ee : rbeg) * A.H + h;
      if (ee < rend && A.hvec && h + 3 < A.H) {
        hv[s] = __ldg(reinterpret_cast<const float4*>(src));
      } else {
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = (ee < rend && h + k < A.H) ? __ldg(src + k) : 0.f;
        hv[s] = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
  };
  auto stash = [&](int buf) {
    float out[8];
    gw8_compute<D1, D3>(r, c, out);
#pragma unroll
    for (int i = 0; i < 8; ++i) bsum[i] += out[i];
    *reinterpret_cast<float4*>(&gwt[buf][ge][go * 8]) = make_float4(out[0], out[1], out[2], out[3]);
    *reinterpret_cast<float4*>(&gwt[buf][ge][go * 8 + 4]) =
        make_float4(out[4], out[5], out[6], out[7]);
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int q = tid + s * 128;
      *reinterpret_cast<float4*>(&ht[buf][q >> 4][(q & 15) * 4]) = hv[s];
    }
  };
  const int64_t nsteps = rend > rbeg ? (rend - rbeg + kDaE - 1) / kDaE : 0;
  if (nsteps > 0) {
    fetch(rbeg);
    stash(0);
  }
  __syncthreads();
  for (int64_t step = 0; step < nsteps; ++step) {
    const int buf = static_cast<int>(step & 1);
    const bool more = step + 1 < nsteps;
    if (more) fetch(rbeg + (step + 1) * kDaE);
    mma_4x8<kDaE>(gwt[buf], ht[buf], m0, n0, acc);
    if (more) stash(buf ^ 1);
    __syncthreads();
  }
  float* dout = A.da + static_cast<int64_t>(blockIdx.z) * A.da_numel;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int u = ub + m0 + a;
    if (u >= A.U) continue;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int h = hb + n0 + (b & 3) + (b >> 2) * 32;
      if (h < A.H) dout[(static_cast<int64_t>(p) * A.U + u) * A.H + h] = pair_at(acc[a], b);
    }
  }
  if (A.db != nullptr && hb == 0) {
    // sum the per-thread bias partials over the 16 edge lanes, in lane order
#pragma unroll
    for (int i = 0; i < 8; ++i) red[ge * kDaU + go * 8 + i] = bsum[i];
    __syncthreads();
    if (tid < kDaU && ub + tid < A.U) {
      float sum = 0.f;
      for (int k = 0; k < kDaE; ++k) sum += red[k * kDaU + tid];
      A.db[static_cast<int64_t>(blockIdx.z) * A.db_numel + static_cast<int64_t>(p) * A.U + ub +
           tid] = sum;
    }
  }
}

__global__ void __launch_bounds__(128, 4) radial_dalpha(DaArgs A) {
  __shared__ __align__(16) float gwt[2][kDaE][kDaU];
  __shared__ __align__(16) float ht[2][kDaE][kDaH];
  const int4 pt = A.t.paths[blockIdx.x];
  const int d1 = A.t.in1[pt.x].y, d3 = A.t.in1[pt.z].y;
  float* red = &gwt[0][0][0];  // reused after the main loop (kDaE x kDaU floats)
  with_dims(d1, d3, [&]<int D1, int D3>() { radial_dalpha_body<D1, D3>(A, gwt, ht, red); });
}

// ------------------------------------------------------------ materialized gw
//
// radial_gw: gw[e, p*U + u] = sum_{kc,a,b} c_p[kc][a][b] g_k[e,u,kc] x_i[e,u,a] y_j[e,b]
// for one block of edges, written row-major [E][Wn] so that dhidden = gw alpha and
// dalpha = gw^T hidden run as plain GEMMs (sgemm_tile).  A CTA takes 16 edges; per
// path each thread writes 4 consecutive channels of one edge (one float4 store),
// reading x and g through L1 (the CTA's rows are re-read by every path).
constexpr int kGwEdges = 16;

struct GwArgs {
  const float* x; const float* ang; const float* g; float* gw;
  int64_t rows; int U, W1, W2; int64_t Wn; UvuDev t; bool vec;
};

__global__ void __launch_bounds__(256) radial_gw(GwArgs A) {
  extern __shared__ float gys[];  // [kGwEdges][W2]
  const int tid = threadIdx.x;
  const int64_t e0 = static_cast<int64_t>(blockIdx.x) * kGwEdges;
  for (int q = tid; q < kGwEdges * A.W2; q += 256) {
    const int r = q / A.W2, c = q - r * A.W2;
    gys[q] = e0 + r < A.rows ? __ldg(A.ang + (e0 + r) * A.W2 + c) : 0.f;
  }
  __syncthreads();
  const int nuq = (A.U + 3) / 4;                 // channel quads per path
  const int per_path = kGwEdges * nuq;
  for (int p = 0; p < A.t.np; ++p) {
    const int4 pt = A.t.paths[p];
    const int2 ei = A.t.in1[pt.x], ej = A.t.in2[pt.y], ek = A.t.in1[pt.z];
    float c[8];
    load_coef(A.t, p, c);
    for (int q = tid; q < per_path; q += 256) {
      const int r = q / nuq, u0 = (q - r * nuq) * 4;
      const int64_t e = e0 + r;
      if (e >= A.rows) continue;
      const float y0 = gys[r * A.W2 + ej.x], y1 = ej.y == 2 ? gys[r * A.W2 + ej.x + 1] : 0.f;
      const float c00 = fmaf(c[0], y0, c[1] * y1), c01 = fmaf(c[2], y0, c[3] * y1);
      const float c10 = fmaf(c[4], y0, c[5] * y1), c11 = fmaf(c[6], y0, c[7] * y1);
      const float* xs = A.x + e * A.W1 + ei.x + u0 * ei.y;
      const float* gs = A.g + e * A.W1 + ek.x + u0 * ek.y;
      float out[4];
      with_dims(ei.y, ek.y, [&]<int D1, int D3>() {
        float xv[4 * D1], gv[4 * D3];
        ut_like_load<D1>(xv, xs, u0, A.U, A.vec);
        ut_like_load<D3>(gv, gs, u0, A.U, A.vec);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float x0 = xv[k * D1], x1 = D1 == 2 ? xv[k * D1 + 1] : 0.f;
          const float g0 = gv[k * D3], g1 = D3 == 2 ? gv[k * D3 + 1] : 0.f;
          float t0 = c00 * x0;
          if (D1 == 2) t0 = fmaf(c01, x1, t0);
          if (D3 == 2) {
            float t1 = c10 * x0;
            if (D1 == 2) t1 = fmaf(c11, x1, t1);
            out[k] = fmaf(g0, t0, g1 * t1);
          } else {
            out[k] = g0 * t0;
          }
        }
      });
      float* dst = A.gw + e * A.Wn + static_cast<int64_t>(p) * A.U + u0;
      if (A.vec && u0 + 3 < A.U) {
        *reinterpret_cast<float4*>(dst) = make_float4(out[0], out[1], out[2], out[3]);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (u0 + k < A.U) dst[k] = out[k];
      }
    }
  }
}

// Column sums of rows [r0, r1) of a [rows][n] matrix into dst[blockIdx.y][n]
// (row chunks summed in a fixed order by radial_sum_chunks).
__global__ void column_sums(const float* __restrict__ src, float* __restrict__ dst, int64_t rows,
                            int64_t n, int64_t chunk_rows) {
  const int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (col >= n) return;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * chunk_rows;
  const int64_t r1 = r0 + chunk_rows < rows ? r0 + chunk_rows : rows;
  float s = 0.f;
  for (int64_t r = r0; r < r1; ++r) s += src[r * n + col];
  dst[static_cast<int64_t>(blockIdx.y) * n + col] = s;
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
  if (c.M > 32 || c.M2 > 32) return fail(ICTC_ERR_UNSUPPORTED, "m_max above 32");
  return ICTC_OK;
}

// Weight gradients through a materialized gw: edges in blocks of at most
// kGwBlock and at most kGwBlockBytes of gw (but never under kGwMinBlock edges, so
// a block's dx/dy tile launch still fills the GPU), dalpha split over kchunks K
// ranges per block; partials summed in a fixed order at the end.
constexpr int64_t kGwBlock = 262144;
constexpr size_t kGwBlockBytes = size_t(4) << 30;
constexpr int64_t kGwMinBlock = 32768;

struct GwPlan {
  bool ok;
  int64_t blk, nblocks, kchunks, k_chunk;
  size_t gw_bytes, da_part_bytes, db_part_bytes;
};

GwPlan radial_gw_plan(int device, int64_t rows, int64_t Wn, int U, int H) {
  GwPlan g{};
  if (rows <= 0 || Wn % 4 != 0 || U % 4 != 0 || H % 4 != 0) return g;
  // Blocks of whole waves of the dx/dy tile (one CTA per SM, RT edges each),
  // balanced so that about kGwBlockBytes of gw stay live at a time.
  int64_t cap = static_cast<int64_t>(kGwBlockBytes / (static_cast<size_t>(Wn) * sizeof(float)));
  cap = cap < kGwMinBlock ? kGwMinBlock : (cap > kGwBlock ? kGwBlock : cap);
  const int64_t wave = static_cast<int64_t>(sm_count(device)) * (radial_ut(U) == 64 ? 128 : 64);
  const int64_t waves = (rows + wave - 1) / wave;
  const int64_t blocks = (rows + cap - 1) / cap;
  const int64_t blk = ((waves + blocks - 1) / blocks) * wave;
  g.blk = rows < blk ? rows : blk;
  g.nblocks = (rows + g.blk - 1) / g.blk;
  const int64_t tiles = ((Wn + kGemmBM - 1) / kGemmBM) * ((H + kGemmBN - 1) / kGemmBN);
  int64_t kc = (16 * static_cast<int64_t>(sm_count(device)) + tiles - 1) / tiles;
  const int64_t max_kc = (g.blk + 1023) / 1024;
  if (kc > max_kc) kc = max_kc;
  if (kc < 1) kc = 1;
  g.k_chunk = (((g.blk + kc - 1) / kc) + kGemmBK - 1) / kGemmBK * kGemmBK;
  g.kchunks = (g.blk + g.k_chunk - 1) / g.k_chunk;
  g.gw_bytes = static_cast<size_t>(g.blk) * Wn * sizeof(float);
  g.da_part_bytes = static_cast<size_t>(g.nblocks * g.kchunks) * Wn * H * sizeof(float);
  g.db_part_bytes = static_cast<size_t>(g.nblocks * g.kchunks) * Wn * sizeof(float);
  g.ok = true;
  return g;
}

int64_t radial_chunks(int device, int64_t rows, int P, int U, int H) {
  const int64_t tiles = static_cast<int64_t>(P) * ((U + kDaU - 1) / kDaU) * ((H + kDaH - 1) / kDaH);
  int64_t chunks = (8 * sm_count(device) + tiles - 1) / tiles;
  const int64_t max_chunks = (rows + 1023) / 1024;
  if (chunks > max_chunks) chunks = max_chunks;
  return chunks < 1 ? 1 : chunks;
}

}  // namespace

int radial_take_device_error(int* code) {
  cudaError_t e;
  if (take_unit_device_error(code, &e) != 0) return cuda_fail(e, "radial device error flag");
  return ICTC_OK;
}

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
  const size_t at = radial_at_bytes(P, c.U, c.H);
  if (rows <= 0) {
    *forward_bytes = 0;
    *backward_bytes = 0;
    return ICTC_OK;
  }
  const int64_t chunks = radial_chunks(device, rows, static_cast<int>(P), c.U, c.H);
  const size_t Wn = static_cast<size_t>(P) * c.U;
  size_t part = chunks > 1 ? static_cast<size_t>(chunks) * (Wn * c.H + Wn) * sizeof(float) : 0;
  const GwPlan gp = radial_gw_plan(device, rows, static_cast<int64_t>(Wn), c.U, c.H);
  if (gp.ok) {
    const size_t gwb = gp.gw_bytes + gp.da_part_bytes + gp.db_part_bytes;
    if (gwb > part) part = gwb;
  }
  *forward_bytes = at;
  *backward_bytes = at + part;
  return ICTC_OK;
}

namespace {

// Forward over rows of `left`, or, with `xrow`, over rows xrow[e] of `left` (which
// then has xrows rows): only the edge tile reads gathered rows, so a configuration
// that needs the row tile answers ICTC_ERR_UNSUPPORTED there.
int32_t radial_forward_impl(const float* left, const int64_t* xrow, int64_t xrows,
                            const float* angular, const float* radial_hidden,
                            const float* alpha, const float* bias, float* output, int64_t rows,
                            ICTC_RADIAL_ARGS, const void* device_table, void* workspace,
                            size_t workspace_bytes, void* stream) {
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
  const size_t need = radial_at_bytes(l.np, c.U, c.H);
  if (workspace_bytes < need || !workspace || !aligned(workspace, 16))
    return fail(ICTC_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu (16-byte aligned)",
                workspace_bytes, need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* at = static_cast<float*>(workspace);
  const bool tile = radial_tile_fits(c.U, c.H, th.width2, l.np, l.n1, l.n2, false);
  if (tile)
    transpose_alpha<<<1024, 256, 0, s>>>(alpha, at, l.np, c.U, radial_ut(c.U),
                                         radial_tiles(c.U), c.H);
  else
    transpose_alpha<<<1024, 256, 0, s>>>(alpha, at, l.np, c.U, Up, 1, c.H);
  const UvuDev t = radial_dev(device_table, l);
  const bool vec = (th.width1 % 4 == 0) && (c.U % 4 == 0) && aligned(left, 16) &&
                   aligned(output, 16);
  RadTileArgs ra{left, nullptr, radial_hidden, angular, at, bias, output, nullptr, rows,
                 c.U, Up, c.H, th.width1, th.width2, t, vec};
  ra.xrow = xrow;
  ra.xrows = xrows;
  st = launch_radial_tile<kRtFwd>(ra, s);
  if (st == ICTC_ERR_UNSUPPORTED && xrow != nullptr)
    return fail(ICTC_ERR_UNSUPPORTED,
                "gathered radial forward: hidden width %d does not fit the edge tile", c.H);
  if (st == ICTC_ERR_UNSUPPORTED) {
    // hidden tile too large to stay resident: the generic row tile streams it
    RowtileArgs rr{left, nullptr, radial_hidden, angular, at, bias, output, nullptr, rows,
                   c.U, Up, c.H, th.width1, c.H, th.width2, t};
    st = launch_rowtile<kRadFwd>(rr, s);
  }
  return st;
}

// Backward; with `xrow` (gathered first input) only the edge tile and the
// edge-weight-gradient GEMMs run, so a request they do not cover (no dx / dy
// requested while dalpha, dbias or dhidden are, or a hidden width the edge tile
// cannot hold) answers ICTC_ERR_UNSUPPORTED.
int32_t radial_backward_impl(
    const float* left, const int64_t* xrow, int64_t xrows, const float* angular,
    const float* radial_hidden, const float* alpha, const float* bias, const float* grad_output,
    float* grad_left, float* grad_angular, float* grad_hidden, float* grad_alpha,
    float* grad_bias, int64_t rows, ICTC_RADIAL_ARGS, int32_t needed, const void* device_table,
    void* workspace, size_t workspace_bytes, void* stream) {
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
  const size_t at_bytes = radial_at_bytes(l.np, c.U, c.H);
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
  const GwPlan gp = radial_gw_plan(device, rows, Wn, c.U, c.H);
  const bool gw_path = (needed & 28) && gp.ok && aligned(alpha, 16) && aligned(radial_hidden, 16) &&
                       (!(needed & 4) || aligned(grad_hidden, 16)) &&
                       workspace_bytes >= at_bytes + gp.gw_bytes + gp.da_part_bytes +
                                              gp.db_part_bytes;
  const bool tvec = (W1 % 4 == 0) && (c.U % 4 == 0) && aligned(left, 16) &&
                    aligned(grad_output, 16) && aligned(grad_left, 16);
  if (xrow != nullptr &&
      (!(needed & 3) || ((needed & 28) && !gw_path) ||
       !radial_tile_fits(c.U, c.H, W2, l.np, l.n1, l.n2, true)))
    return fail(ICTC_ERR_UNSUPPORTED,
                "gathered radial backward covers dx / dy requests on the edge tile only");
  if (needed & 3) {
    // dx and dy together: both need the regenerated edge weights
    if (radial_tile_fits(c.U, c.H, W2, l.np, l.n1, l.n2, true))
      transpose_alpha<<<1024, 256, 0, s>>>(alpha, at, l.np, c.U, radial_ut(c.U),
                                           radial_tiles(c.U), c.H);
    else
      transpose_alpha<<<1024, 256, 0, s>>>(alpha, at, l.np, c.U, Up, 1, c.H);
    // scratch outputs when only one of dx / dy is requested are not allowed to
    // alias inputs; the caller passes both buffers (see the Python wrapper)
    if (!grad_left || !grad_angular)
      return fail(ICTC_ERR_INVALID, "dx and dy buffers are both required when either is");
    if (!gw_path) {
      RadTileArgs ra{grad_output, left, radial_hidden, angular, at, bias, grad_left,
                     grad_angular, rows, c.U, Up, c.H, W1, W2, t, tvec};
      ra.xrow = xrow;
      ra.xrows = xrows;
      st = launch_radial_tile<kRtDx>(ra, s);
      if (st == ICTC_ERR_UNSUPPORTED) {
        if (c.U > kUT)
          return fail(ICTC_ERR_UNSUPPORTED,
                      "radial dx/dy: hidden width %d with more than %d channels does not fit the "
                      "edge tile", c.H, kUT);
        RowtileArgs rr{grad_output, left, radial_hidden, angular, at, bias, grad_left,
                       grad_angular, rows, c.U, Up, c.H, W1, c.H, W2, t};
        st = launch_rowtile<kRadDx>(rr, s);
      }
      if (st != ICTC_OK) return st;
    }
  }
  if (gw_path) {
    // gw blocks in the workspace, then dhidden = gw alpha and dalpha = gw^T hidden
    float* gw = partial;
    float* dapart = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(gw) + gp.gw_bytes);
    float* dbpart =
        reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(dapart) + gp.da_part_bytes);
    const bool gvec = (W1 % 4 == 0) && aligned(left, 16) && aligned(grad_output, 16);
    const int64_t nparts = gp.nblocks * gp.kchunks;
    for (int64_t blk = 0; blk < gp.nblocks; ++blk) {
      const int64_t r0 = blk * gp.blk;
      const int64_t nb = rows - r0 < gp.blk ? rows - r0 : gp.blk;
      bool gw_done = false;
      if (needed & 3) {
        // dx, dy of the block; the tile also writes the block's gw
        RadTileArgs ra{grad_output + r0 * W1, xrow ? left : left + r0 * W1,
                       radial_hidden + r0 * c.H, angular + r0 * W2, at, bias,
                       grad_left + r0 * W1, grad_angular + r0 * W2, nb, c.U, Up, c.H, W1, W2, t,
                       tvec};
        ra.gw = gw;
        ra.Wn = Wn;
        ra.xrow = xrow ? xrow + r0 : nullptr;
        ra.xrows = xrows;
        st = launch_radial_tile<kRtDx>(ra, s);
        if (st == ICTC_ERR_UNSUPPORTED) {  // hidden tile too large: row tile, gw separately
          if (c.U > kUT)
            return fail(ICTC_ERR_UNSUPPORTED,
                        "radial dx/dy: hidden width %d with more than %d channels does not fit "
                        "the edge tile", c.H, kUT);
          RowtileArgs rr{grad_output + r0 * W1, left + r0 * W1, radial_hidden + r0 * c.H,
                         angular + r0 * W2, at, bias, grad_left + r0 * W1,
                         grad_angular + r0 * W2, nb, c.U, Up, c.H, W1, c.H, W2, t};
          st = launch_rowtile<kRadDx>(rr, s);
        } else {
          gw_done = st == ICTC_OK;
        }
        if (st != ICTC_OK) return st;
      }
      if (!gw_done) {
        GwArgs ga{left + r0 * W1, angular + r0 * W2, grad_output + r0 * W1, gw, nb, c.U, W1, W2,
                  Wn, t, gvec};
        radial_gw<<<static_cast<unsigned>(ceil_div(nb, kGwEdges)), 256,
                    static_cast<size_t>(kGwEdges) * W2 * sizeof(float), s>>>(ga);
      }
      if (needed & 4) {
        SgemmArgs g{gw, alpha, grad_hidden + r0 * c.H, nb, c.H, Wn, Wn, c.H, c.H, Wn, 0};
        const dim3 grid(static_cast<unsigned>(ceil_div(nb, kGemmBM)),
                        static_cast<unsigned>(ceil_div(c.H, kGemmBN)), 1);
        sgemm_tile<false><<<grid, kGemmThreads, 0, s>>>(g);
      }
      if (needed & 8) {
        SgemmArgs g{gw, radial_hidden + r0 * c.H, dapart + blk * gp.kchunks * Wn * c.H, Wn, c.H,
                    nb, Wn, c.H, c.H, gp.k_chunk, Wn * c.H};
        const dim3 grid(static_cast<unsigned>(ceil_div(Wn, kGemmBM)),
                        static_cast<unsigned>(ceil_div(c.H, kGemmBN)),
                        static_cast<unsigned>(ceil_div(nb, gp.k_chunk)));
        sgemm_tile<true><<<grid, kGemmThreads, 0, s>>>(g);
      }
      if (needed & 16) {
        const dim3 grid(static_cast<unsigned>(ceil_div(Wn, 256)),
                        static_cast<unsigned>(ceil_div(nb, gp.k_chunk)));
        column_sums<<<grid, 256, 0, s>>>(gw, dbpart + blk * gp.kchunks * Wn, nb, Wn, gp.k_chunk);
      }
      // a last block shorter than the others leaves its unused chunks at zero
      const int64_t used = ceil_div(nb, gp.k_chunk);
      if (used < gp.kchunks) {
        if (needed & 8) {
          e = cudaMemsetAsync(dapart + (blk * gp.kchunks + used) * Wn * c.H, 0,
                              static_cast<size_t>(gp.kchunks - used) * Wn * c.H * sizeof(float), s);
          if (e != cudaSuccess) return cuda_fail(e, "memset");
        }
        if (needed & 16) {
          e = cudaMemsetAsync(dbpart + (blk * gp.kchunks + used) * Wn, 0,
                              static_cast<size_t>(gp.kchunks - used) * Wn * sizeof(float), s);
          if (e != cudaSuccess) return cuda_fail(e, "memset");
        }
      }
    }
    if (needed & 8)
      radial_sum_chunks<<<1024, 256, 0, s>>>(dapart, grad_alpha, Wn * c.H,
                                             static_cast<int>(nparts));
    if (needed & 16)
      radial_sum_chunks<<<256, 256, 0, s>>>(dbpart, grad_bias, Wn, static_cast<int>(nparts));
  } else {
    const bool vec = (W1 % 4 == 0) && (c.U % 8 == 0) && aligned(left, 16) && aligned(grad_output, 16);
    if (needed & 4) {
      DhArgs da{left, angular, grad_output, alpha, grad_hidden, rows, c.U, c.H, W1, W2, t, vec,
                (c.H % 4 == 0) && aligned(alpha, 16)};
      const dim3 grid(static_cast<unsigned>(ceil_div(rows, kDhE)), (c.H + kDhH - 1) / kDhH);
      radial_dhidden<<<grid, 128, 0, s>>>(da);
    }
    if (needed & 24) {
      // grad_alpha doubles as scratch when only the bias gradient is requested
      if (!grad_alpha) return fail(ICTC_ERR_INVALID, "grad_alpha is required when dbias is");
      const int64_t chunk_rows = ((ceil_div(rows, chunks) + kDaE - 1) / kDaE) * kDaE;
      const dim3 grid(static_cast<unsigned>(l.np),
                      ((c.U + kDaU - 1) / kDaU) * ((c.H + kDaH - 1) / kDaH),
                      static_cast<unsigned>(chunks));
      const int64_t da_numel = Wn * c.H;
      float* da = chunks > 1 ? partial : grad_alpha;
      float* db = chunks > 1 ? partial + chunks * da_numel : ((needed & 16) ? grad_bias : nullptr);
      DaArgs aa{left, angular, grad_output, radial_hidden, da, db, rows, chunk_rows, da_numel, Wn,
                c.U, c.H, W1, W2, t, vec, (c.H % 4 == 0) && aligned(radial_hidden, 16)};
      radial_dalpha<<<grid, 128, 0, s>>>(aa);
      if (chunks > 1) {
        radial_sum_chunks<<<1024, 256, 0, s>>>(partial, grad_alpha, da_numel,
                                               static_cast<int>(chunks));
        if (needed & 16)
          radial_sum_chunks<<<256, 256, 0, s>>>(partial + chunks * da_numel, grad_bias, Wn,
                                                static_cast<int>(chunks));
      }
    }
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "radial backward launch");
}

}  // namespace

extern "C" int32_t ictc_o2_radial_forward(const float* left, const float* angular,
                                          const float* radial_hidden, const float* alpha,
                                          const float* bias, float* output, int64_t rows,
                                          ICTC_RADIAL_ARGS, const void* device_table,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  return radial_forward_impl(left, nullptr, 0, angular, radial_hidden, alpha, bias, output, rows,
                             channels, m_max, parity, m_max_in2, parity_in2, normalization,
                             path_normalization, hidden, device_table, workspace,
                             workspace_bytes, stream);
}

extern "C" int32_t ictc_o2_radial_backward(
    const float* left, const float* angular, const float* radial_hidden, const float* alpha,
    const float* bias, const float* grad_output, float* grad_left, float* grad_angular,
    float* grad_hidden, float* grad_alpha, float* grad_bias, int64_t rows, ICTC_RADIAL_ARGS,
    int32_t needed, const void* device_table, void* workspace, size_t workspace_bytes,
    void* stream) {
  return radial_backward_impl(left, nullptr, 0, angular, radial_hidden, alpha, bias, grad_output,
                              grad_left, grad_angular, grad_hidden, grad_alpha, grad_bias, rows,
                              channels, m_max, parity, m_max_in2, parity_in2, normalization,
                              path_normalization, hidden, needed, device_table, workspace,
                              workspace_bytes, stream);
}

extern "C" int32_t ictc_o2_radial_forward_gathered(
    const float* nodes, const int64_t* left_index, int64_t node_rows, const float* angular,
    const float* radial_hidden, const float* alpha, const float* bias, float* output,
    int64_t rows, ICTC_RADIAL_ARGS, const void* device_table, void* workspace,
    size_t workspace_bytes, void* stream) {
  if (rows > 0 && (left_index == nullptr || node_rows < 1))
    return fail(ICTC_ERR_INVALID, "left_index and node_rows >= 1 are required");
  return radial_forward_impl(nodes, left_index, node_rows, angular, radial_hidden, alpha, bias,
                             output, rows, channels, m_max, parity, m_max_in2, parity_in2,
                             normalization, path_normalization, hidden, device_table, workspace,
                             workspace_bytes, stream);
}

extern "C" int32_t ictc_o2_radial_backward_gathered(
    const float* nodes, const int64_t* left_index, int64_t node_rows, const float* angular,
    const float* radial_hidden, const float* alpha, const float* bias, const float* grad_output,
    float* grad_left_edges, float* grad_angular, float* grad_hidden, float* grad_alpha,
    float* grad_bias, int64_t rows, ICTC_RADIAL_ARGS, int32_t needed, const void* device_table,
    void* workspace, size_t workspace_bytes, void* stream) {
  if (rows > 0 && (left_index == nullptr || node_rows < 1))
    return fail(ICTC_ERR_INVALID, "left_index and node_rows >= 1 are required");
  return radial_backward_impl(nodes, left_index, node_rows, angular, radial_hidden, alpha, bias,
                              grad_output, grad_left_edges, grad_angular, grad_hidden, grad_alpha,
                              grad_bias, rows, channels, m_max, parity, m_max_in2, parity_in2,
                              normalization, path_normalization, hidden, needed, device_table,
                              workspace, workspace_bytes, stream);
}
