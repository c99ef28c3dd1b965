// Shared-weight uvu dy: uvu_dy_stage.
//
//   dy_j[r,v,b] = sum_{p: j_p = j} sum_u w_p[u,v] s_p[r,u,b],
//   s_p[r,u,b]  = sum_{kc,a} c_p[kc][a][b] g_k[r,u,kc] x_i[r,u,a]
//
// A CTA (256 threads) owns 16 rows and walks the paths grouped by second entry
// j.  For each path the slices x_i[16 rows][U d1], g_k[16 rows][U d3] and the
// weights w_p[U][V] arrive by cp.async one path ahead; s_p is built from shared
// memory into S[u][(row, b)] and then contracted over u (GEMM: an 8 (row, b) x 4 v
// tile per thread; warp w takes the channels u = w + 8 i; the eight warps' sums are
// added in a fixed order, a three-round tree, when the j group ends).  For a
// one-component y_j the GEMM skips the b = 1 entries, whose sums are never stored.
// Needs U <= 128, V <= 32 and 16-byte aligned rows; other shapes use uvu_dy_tile.
//
// This header is included inside the anonymous namespace of uvu_kernels.cu.
#pragma once

constexpr int kDyRows = 16;
constexpr int kDyU = 128;
constexpr int kDyV = 32;
constexpr int kDyLd = 2 * kDyRows + 4;  // S row stride (floats): 32 (row, b) + pad
constexpr int kDyLdW = kDyV + 4;        // weight row stride (floats)
constexpr int kDySx = 2 * kDyU + 16;    // slice row stride: conflict-free s generation reads

struct DyArgs {
  const float* x; const float* g; const float* w; float* dy;
  int64_t rows;
  int U, V, W1, W2;
  UvuDev t;
};

// About 102 KB: two CTAs per SM.  x / g slices are single-buffered (the next path's
// slices are copied while this path's GEMM runs, after S has been built from
// them); the weights are double-buffered.
struct DySmem {
  float xs[kDyRows][kDySx];
  float gs[kDyRows][kDySx];
  float wp[2][kDyU][kDyLdW];
  float S[kDyU][kDyLd];
  float red[4][32][32];  // warp-sum tree: [warp][value][lane]
};

// Path record of path position pos (by_j order), built once per CTA after DySmem in
// shared memory, so the per-path reads are shared-memory loads rather than a chain of
// dependent global loads: {path, x_i offset, g_k offset, y_j offset | dims | last of j},
// the dims d1 - 1, d3 - 1, d2 - 1 in bits 24-26 and "last path of its j group" in
// bit 27 of the fourth word (y_j offsets are below 2^24); then the path's 8
// coefficients.
struct DyPath {
  int4 rec;
  float2 c[4];
};

inline size_t uvu_dy_stage_smem(int np) {
  return sizeof(DySmem) + static_cast<size_t>(np) * sizeof(DyPath);
}

inline bool uvu_dy_stage_fits(int U, int V, int W1, bool aligned_rows) {
  return U <= kDyU && V <= kDyV && U % 4 == 0 && V % 4 == 0 && W1 % 4 == 0 && aligned_rows;
}

__device__ __forceinline__ void dy_cp16(void* smem, const void* gmem, bool valid) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}

// Both components of a staged one- or two-component slot (the second is 0 for
// one-component entries); one 8-byte access for two-component slots keeps the
// lanes of consecutive channels on distinct banks.
__device__ __forceinline__ float2 dy_slot(const float* p, int dim) {
  return dim == 2 ? *reinterpret_cast<const float2*>(p) : make_float2(p[0], 0.f);
}

__global__ void __launch_bounds__(256, 2) uvu_dy_stage(DyArgs A) {
  extern __shared__ __align__(16) unsigned char dy_raw[];
  DySmem& S = *reinterpret_cast<DySmem*>(dy_raw);
  DyPath* recs = reinterpret_cast<DyPath*>(dy_raw + sizeof(DySmem));
  const int tid = threadIdx.x;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kDyRows;
  const int nvalid = A.rows - row0 < kDyRows ? static_cast<int>(A.rows - row0) : kDyRows;
  const int np = A.t.np;
  for (int q = tid; q < np; q += 256) {
    const int p = A.t.by_j[q];
    const int4 pt = A.t.paths[p];
    const int2 ei = A.t.in1[pt.x], ej = A.t.in2[pt.y], ek = A.t.in1[pt.z];
    const bool last = q + 1 == np || A.t.paths[A.t.by_j[q + 1]].y != pt.y;
    DyPath d;
    d.rec = make_int4(p, ei.x, ek.x,
                      ej.x | ((ei.y - 1) << 24) | ((ek.y - 1) << 25) | ((ej.y - 1) << 26) |
                          (last ? 1 << 27 : 0));
    const float2* cp = reinterpret_cast<const float2*>(A.t.coef + 8 * p);
#pragma unroll
    for (int k = 0; k < 4; ++k) d.c[k] = __ldg(cp + k);
    recs[q] = d;
  }
  __syncthreads();  // path records visible
  // x / g slices of path position pos (zero-filled past the rows)
  auto issue_xg = [&](int pos) {
    if (pos < np) {
      const int4 rc = recs[pos].rec;
      const int2 ei = make_int2(rc.y, ((rc.w >> 24) & 1) + 1);
      const int2 ek = make_int2(rc.z, ((rc.w >> 25) & 1) + 1);
      const int nx = A.U * ei.y / 4, ng = A.U * ek.y / 4;  // float4 per row (<= 64)
      // thread -> float4 column tid % 64 of rows tid / 64 + 4 k: no index division
      const int c = tid & 63, rb = tid >> 6;
#pragma unroll
      for (int k = 0; k < kDyRows / 4; ++k) {
        const int r = rb + 4 * k;
        const bool ok = r < nvalid;
        if (c < nx)
          dy_cp16(&S.xs[r][c * 4], ok ? A.x + (row0 + r) * A.W1 + ei.x + c * 4 : A.x, ok);
        if (c < ng)
          dy_cp16(&S.gs[r][c * 4], ok ? A.g + (row0 + r) * A.W1 + ek.x + c * 4 : A.g, ok);
      }
    }
  };
  // weights w_p [U][V] of path position pos into buffer buf
  auto issue_w = [&](int pos, int buf) {
    if (pos < np) {
      const int p = recs[pos].rec.x;
      const float* wsrc = A.w + static_cast<int64_t>(p) * A.U * A.V;
      // thread -> float4 column tid % 8 of channels tid / 8 + 32 k (V <= 32, U <= 128)
      const int c = tid & 7, ub = tid >> 3;
      if (4 * c < A.V) {
#pragma unroll
        for (int k = 0; k < kDyU / 32; ++k) {
          const int u = ub + 32 * k;
          if (u < A.U) dy_cp16(&S.wp[buf][u][4 * c], wsrc + u * A.V + 4 * c, true);
        }
      }
    }
  };
  // zero the parts of the buffers that copies do not cover (channels >= U, v >= V)
  for (int q = tid; q < kDyRows * kDySx; q += 256) {
    (&S.xs[0][0])[q] = 0.f;
    (&S.gs[0][0])[q] = 0.f;
  }
  for (int q = tid; q < 2 * kDyU * kDyLdW; q += 256) (&S.wp[0][0][0])[q] = 0.f;
  __syncthreads();
  issue_xg(0);
  issue_w(0, 0);
  asm volatile("cp.async.commit_group;" ::: "memory");
  // generation: channel 8 (warp + 8 (k & 1)) + lane % 8, row 4 (k / 2) + lane / 8 (a
  // half warp stores 8 channels x 2 rows: conflict-free float2 stores)
  const int lane = tid & 31, warp = tid >> 5;
  // GEMM: channels u = warp + 8 i, (row, b) octet ro, v quad vq
  const int ro = lane >> 3, vq = lane & 7;
  float2 acc[8][2];  // [(row, b)][v pair]
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b) acc[a][b] = make_float2(0.f, 0.f);
  for (int pos = 0; pos < np; ++pos) {
    const int buf = pos & 1;
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // slices of pos visible; previous GEMM done with S and wp[buf ^ 1]
    const int4 rc = recs[pos].rec;
    const int2 ei = make_int2(rc.y, ((rc.w >> 24) & 1) + 1);
    const int2 ek = make_int2(rc.z, ((rc.w >> 25) & 1) + 1);
    const int2 ej = make_int2(rc.w & 0xffffff, ((rc.w >> 26) & 1) + 1);
    // coefficient pairs over b: (c[4 kc + 2 a], c[4 kc + 2 a + 1])
    const float2 c0 = recs[pos].c[0], c1 = recs[pos].c[1], c2 = recs[pos].c[2],
                 c3 = recs[pos].c[3];
    // (s0, s1) = g0 (c0 x0 + c1 x1) + g1 (c2 x0 + c3 x1), both b at once (f32x2)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int u = 8 * (warp + 8 * (k & 1)) + (lane & 7);
      const int r = 4 * (k >> 1) + (lane >> 3);
      const float2 xv = dy_slot(&S.xs[r][u * ei.y], ei.y);
      const float2 gv = dy_slot(&S.gs[r][u * ek.y], ek.y);
      const float2 t0 = fma2(xv.y, c1, __fmul2_rn(make_float2(xv.x, xv.x), c0));
      const float2 t1 = fma2(xv.y, c3, __fmul2_rn(make_float2(xv.x, xv.x), c2));
      *reinterpret_cast<float2*>(&S.S[u][2 * r]) =
          fma2(gv.y, t1, __fmul2_rn(make_float2(gv.x, gv.x), t0));
    }
    __syncthreads();  // S built; x / g free for the next path
    issue_xg(pos + 1);
    issue_w(pos + 1, buf ^ 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    // dy[(r,b)][v] += sum_u S[u][(r,b)] w[u][v] over this warp's channels; for a
    // one-component y_j only the b = 0 entries (even m), whose sums are stored
    auto gemm = [&](auto two) {
      constexpr int MS = decltype(two)::value ? 1 : 2;  // m stride
#pragma unroll 8
      for (int i = 0; i < kDyU / 8; ++i) {
        const int u = warp + 8 * i;
        const float4 a0 = *reinterpret_cast<const float4*>(&S.S[u][8 * ro]);
        const float4 a1 = *reinterpret_cast<const float4*>(&S.S[u][8 * ro + 4]);
        const float4 b4 = *reinterpret_cast<const float4*>(&S.wp[buf][u][4 * vq]);
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float2 bv[2] = {make_float2(b4.x, b4.y), make_float2(b4.z, b4.w)};
#pragma unroll
        for (int m = 0; m < 8; m += MS)
#pragma unroll
          for (int k = 0; k < 2; ++k) acc[m][k] = fma2(av[m], bv[k], acc[m][k]);
      }
    };
    if (ej.y == 2) {
      gemm(std::true_type{});
    } else {
      gemm(std::false_type{});
    }
    const bool last = (rc.w >> 27) & 1;
    if (last) {
      // sum the eight warps in a fixed order: w + 4, w + 2, w + 1 into w
#pragma unroll
      for (int half = 4; half >= 1; half >>= 1) {
        if (warp >= half && warp < 2 * half) {
#pragma unroll
          for (int m = 0; m < 8; ++m)
#pragma unroll
            for (int k = 0; k < 4; ++k) S.red[warp - half][m * 4 + k][lane] = pair_at(acc[m], k);
        }
        __syncthreads();
        if (warp < half) {
#pragma unroll
          for (int m = 0; m < 8; ++m)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              acc[m][k].x += S.red[warp][m * 4 + 2 * k][lane];
              acc[m][k].y += S.red[warp][m * 4 + 2 * k + 1][lane];
            }
        }
        __syncthreads();
      }
      if (warp == 0) {
        // (r, b) = 8 ro + m: row 4 ro + m / 2, component m % 2; v = 4 vq + k
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int r = 4 * ro + (m >> 1), b = m & 1;
          const int64_t row = row0 + r;
          if (row < A.rows && b < ej.y) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int v = 4 * vq + k;
              if (v < A.V) A.dy[row * A.W2 + ej.x + v * ej.y + b] = pair_at(acc[m], k);
            }
          }
        }
      }
#pragma unroll
      for (int m = 0; m < 8; ++m)
#pragma unroll
        for (int k = 0; k < 2; ++k) acc[m][k] = make_float2(0.f, 0.f);
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}
