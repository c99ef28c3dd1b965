// Shared-weight uvu dw: uvu_dw_stage.
//
//   dw_p[u,v] = sum_r sum_b s_p[r,u,b] y_j[r,v,b],
//   s_p[r,u,b] = sum_{kc,a} c_p[kc][a][b] g_k[r,u,kc] x_i[r,u,a]
//
// A CTA (256 threads) owns one path and one chunk of rows.  It walks the rows in
// steps of 16 (about 100 KB of shared memory, two CTAs per SM): the slices x_i,
// g_k [16 rows][U d] and y_j [16 rows][V d2] arrive by cp.async one step ahead
// (double buffer); s is built from shared memory into S[u][(row, b)] and y into
// Y[(row, b)][v]; then the GEMM over K = (row, b) accumulates dw_p.  Each thread
// holds an 8 u x 8 v tile (channels uo + 16 i, v = 8 vo .. 8 vo + 7) over a quarter of
// each step's 32 (row, b) values; the four quarters are summed in a fixed order at
// the end.  Chunks are summed in a fixed order afterwards.  A one-component y_j
// (scalar second-input entry) has no b = 1 terms: its GEMM runs over the b = 0 half of
// K only.  Needs U <= 128, V <= 32 and 16-byte aligned rows.
//
// This header is included inside the anonymous namespace of uvu_kernels.cu.
#pragma once

constexpr int kDwRows = 16;
constexpr int kDwU = 128;
constexpr int kDwV = 32;
constexpr int kDwSx = 2 * kDwU + 16;     // slice row stride: conflict-free s generation reads
constexpr int kDwLdS = 2 * kDwRows + 4;  // S row stride (floats)
constexpr int kDwLdY = kDwV + 4;         // Y row stride (floats)

struct DwArgs {
  const float* x; const float* y; const float* g; float* dst;  // dst: [chunks][Wn]
  int64_t rows, chunk_rows, Wn;
  int U, V, W1, W2;
  UvuDev t;
};

struct DwSmem {
  float xs[2][kDwRows][kDwSx];
  float gs[2][kDwRows][kDwSx];
  float ys[2][kDwRows][kDwV * 2];
  float S[kDwU][kDwLdS];
  float Y[2 * kDwRows][kDwLdY];
};
// K-quarter sums parked for the final reduction: [quarter 1..3][value][thread], in
// the x / g slice area once every step is done.
static_assert(3 * 64 * 64 * sizeof(float) <= 2 * sizeof(float) * 2 * kDwRows * kDwSx,
              "quarter sums must fit the slice buffers");

inline bool uvu_dw_stage_fits(int U, int V, int W1, int W2, bool aligned_rows) {
  return U <= kDwU && V <= kDwV && U % 4 == 0 && V % 4 == 0 && W1 % 4 == 0 && W2 % 4 == 0 &&
         aligned_rows;
}

__global__ void __launch_bounds__(256, 2) uvu_dw_stage(DwArgs A) {
  extern __shared__ __align__(16) unsigned char dw_raw[];
  DwSmem& S = *reinterpret_cast<DwSmem*>(dw_raw);
  const int tid = threadIdx.x;
  const int p = blockIdx.x;
  const int4 pt = A.t.paths[p];
  const int2 ei = A.t.in1[pt.x], ej = A.t.in2[pt.y], ek = A.t.in1[pt.z];
  // coefficient pairs over b: (c[4 kc + 2 a], c[4 kc + 2 a + 1])
  const float2* cp = reinterpret_cast<const float2*>(A.t.coef + 8 * p);
  const float2 c0 = __ldg(cp), c1 = __ldg(cp + 1), c2 = __ldg(cp + 2), c3 = __ldg(cp + 3);
  const int64_t rbeg = static_cast<int64_t>(blockIdx.y) * A.chunk_rows;
  const int64_t rend = rbeg + A.chunk_rows < A.rows ? rbeg + A.chunk_rows : A.rows;
  const int64_t nsteps = rend > rbeg ? (rend - rbeg + kDwRows - 1) / kDwRows : 0;
  const int nx = A.U * ei.y / 4, ng = A.U * ek.y / 4, ny = A.V * ej.y / 4;  // float4 per row
  auto issue = [&](int64_t step, int buf) {
    if (step < nsteps) {
      const int64_t r0 = rbeg + step * kDwRows;
      const int nv = rend - r0 < kDwRows ? static_cast<int>(rend - r0) : kDwRows;
      // thread -> float4 column tid % 64 of rows tid / 64 + 4 k (x, g: <= 64 columns)
      // and column tid % 16 of row tid / 16 (y: <= 16 columns): no index division
      const int cc = tid & 63, rb = tid >> 6;
#pragma unroll
      for (int k = 0; k < kDwRows / 4; ++k) {
        const int r = rb + 4 * k;
        const bool ok = r < nv;
        if (cc < nx)
          dy_cp16(&S.xs[buf][r][cc * 4], ok ? A.x + (r0 + r) * A.W1 + ei.x + cc * 4 : A.x, ok);
        if (cc < ng)
          dy_cp16(&S.gs[buf][r][cc * 4], ok ? A.g + (r0 + r) * A.W1 + ek.x + cc * 4 : A.g, ok);
      }
      const int yc = tid & 15, yr = tid >> 4;
      if (yc < ny) {
        const bool ok = yr < nv;
        dy_cp16(&S.ys[buf][yr][yc * 4], ok ? A.y + (r0 + yr) * A.W2 + ej.x + yc * 4 : A.y, ok);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int q = tid; q < 2 * kDwRows * kDwSx; q += 256) {
    (&S.xs[0][0][0])[q] = 0.f;
    (&S.gs[0][0][0])[q] = 0.f;
  }
  for (int q = tid; q < 2 * kDwRows * kDwV * 2; q += 256) (&S.ys[0][0][0])[q] = 0.f;
  __syncthreads();
  issue(0, 0);
  // generation: channel 8 (warp + 8 (k & 1)) + lane % 8, row 4 (k / 2) + lane / 8 (a
  // half warp stores 8 channels x 2 rows: conflict-free float2 stores)
  const int lane = tid & 31, warp = tid >> 5;
  // GEMM: K quarter kq, channels uo + 16 i, v octet vo (v = 8 vo .. 8 vo + 7)
  const int kq = tid >> 6, uo = (tid & 63) >> 2, vo = tid & 3;
  float2 acc[8][4];  // [channel][v pair]
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = make_float2(0.f, 0.f);
  for (int64_t step = 0; step < nsteps; ++step) {
    const int buf = static_cast<int>(step & 1);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // slices of step visible; previous GEMM done with S and Y
    issue(step + 1, buf ^ 1);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int u = 8 * (warp + 8 * (k & 1)) + (lane & 7);
      const int r = 4 * (k >> 1) + (lane >> 3);
      const float2 xv = dy_slot(&S.xs[buf][r][u * ei.y], ei.y);
      const float2 gv = dy_slot(&S.gs[buf][r][u * ek.y], ek.y);
      // (s0, s1) = g0 (c0 x0 + c1 x1) + g1 (c2 x0 + c3 x1), both b at once (f32x2)
      const float2 t0 = fma2(xv.y, c1, __fmul2_rn(make_float2(xv.x, xv.x), c0));
      const float2 t1 = fma2(xv.y, c3, __fmul2_rn(make_float2(xv.x, xv.x), c2));
      *reinterpret_cast<float2*>(&S.S[u][2 * r]) =
          fma2(gv.y, t1, __fmul2_rn(make_float2(gv.x, gv.x), t0));
    }
    // Y[(r, b)][v] = y_j[r, v, b] for b < d2.  The slice columns past V d2 and the
    // rows past the chunk are zero (zero fill), so Y is zero there too.  A
    // one-component y_j leaves the b = 1 rows of Y unused: its GEMM skips them.
    if (ej.y == 2) {
      // one float4 (v pair x b pair) per thread: 16 rows x 16 pairs
      const int r = tid >> 4, vp = tid & 15;
      const float4 q = *reinterpret_cast<const float4*>(&S.ys[buf][r][4 * vp]);
      *reinterpret_cast<float2*>(&S.Y[2 * r][2 * vp]) = make_float2(q.x, q.z);
      *reinterpret_cast<float2*>(&S.Y[2 * r + 1][2 * vp]) = make_float2(q.y, q.w);
    } else if (tid < kDwRows * kDwV / 4) {
      const int r = tid >> 3, vq = tid & 7;
      *reinterpret_cast<float4*>(&S.Y[2 * r][4 * vq]) =
          *reinterpret_cast<const float4*>(&S.ys[buf][r][4 * vq]);
    }
    __syncthreads();
    // this quarter's 8 (row, b) values, two at a time; b = 1 (kk = 1) only for a
    // two-component y_j (otherwise its terms are s x 0 and leave dw unchanged)
    auto gemm = [&](auto two) {
      constexpr int NKK = decltype(two)::value ? 2 : 1;
#pragma unroll 2
      for (int k0 = 8 * kq; k0 < 8 * kq + 8; k0 += 2) {
        float2 sa[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          sa[i] = *reinterpret_cast<const float2*>(&S.S[uo + 16 * i][k0]);
        float4 yb[NKK][2];
#pragma unroll
        for (int kk = 0; kk < NKK; ++kk)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            yb[kk][h] = *reinterpret_cast<const float4*>(&S.Y[k0 + kk][8 * vo + 4 * h]);
#pragma unroll
        for (int kk = 0; kk < NKK; ++kk) {
          const float2 bv[4] = {make_float2(yb[kk][0].x, yb[kk][0].y),
                                make_float2(yb[kk][0].z, yb[kk][0].w),
                                make_float2(yb[kk][1].x, yb[kk][1].y),
                                make_float2(yb[kk][1].z, yb[kk][1].w)};
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float a = kk == 0 ? sa[i].x : sa[i].y;
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fma2(a, bv[j], acc[i][j]);
          }
        }
      }
    };
    if (ej.y == 2) {
      gemm(std::true_type{});
    } else {
      gemm(std::false_type{});
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  // sum the K quarters in order: quarters 1..3 park their tiles, quarter 0 adds them
  __syncthreads();  // every thread is done with the slice buffers
  float* red = &S.xs[0][0][0];  // [3][64 values][64 threads]
  const int t64 = tid & 63;
  if (kq > 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) red[((kq - 1) * 64 + i * 8 + j) * 64 + t64] = pair_at(acc[i], j);
  }
  __syncthreads();
  if (kq == 0) {
    float* out =
        A.dst + static_cast<int64_t>(blockIdx.y) * A.Wn + static_cast<int64_t>(p) * A.U * A.V;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int u = uo + 16 * i;
      float sum[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sum[j] = pair_at(acc[i], j);
#pragma unroll
        for (int q = 0; q < 3; ++q) sum[j] += red[(q * 64 + i * 8 + j) * 64 + t64];
      }
      if (u < A.U) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int v = 8 * vo + j;
          if (v < A.V) out[static_cast<int64_t>(u) * A.V + v] = sum[j];
        }
      }
    }
  }
}
