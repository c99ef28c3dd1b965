// Shared-weight uvu forward and dx: uvu_tile<MODE, UT>.
//
// A CTA owns 64 rows x UT channels u (UT = 128, or 64 for products with at most
// 64 channels) with 16 * UT / 8 threads in 4 row x 8 channel tiles (channels
// tc*4..+3 and UT/2 + tc*4..+3).  The second input of its rows stays in shared
// memory for the whole CTA, transposed to [W2][64 rows].  It walks the paths;
// per path p it forms
//   proj_p[r,u,b] = sum_v w_p[u,v] y_j[r,v,b]                  (GEMM, K = V)
// with the path's weights [v][u] streaming through a 4-stage bulk-copy ring
// (refilled by the last warp that releases a stage), then couples
//   forward:  out_k[r,u,kc] += sum_{a,b} c[kc][a][b] x_i[r,u,a] proj[b]   (by k)
//   dx:       dx_i[r,u,a]   += sum_{kc,b} c[kc][a][b] g_k[r,u,kc] proj[b] (by i)
// keeping the accumulators of the current k (or i) group in registers.
//
// This header is included inside the anonymous namespace of uvu_kernels.cu.
#pragma once

enum UvuTileMode { kUtFwd = 0, kUtDx = 1 };
constexpr int kUtRows = 64;    // rows per CTA
constexpr int kUtVC = 32;      // v per weight chunk
constexpr int kUtStages = 4;   // weight chunks in flight

struct UvuTileArgs {
  const float* opnd;  // forward: x; dx: g          [rows, W1]
  const float* y;     //                            [rows, W2]
  const float* wt;    // weights as [P][V][Up]
  float* out;         // forward output or dx       [rows, W1]
  int64_t rows;
  int U, Up, V, W1, W2;
  UvuDev t;
  bool vec;  // 16-byte access to 4-channel groups of opnd / out
};

// Thread tiles: 4 rows x NH groups of 4 channels (NH = 2: the 4 x 8 "split" tile;
// NH = 1: the 4 x 4 "wide" tile, twice the threads at half the registers each).
template <int UT, int NH = 2>
struct UtShape {
  static constexpr int TC = UT / (4 * NH);         // threads along the channels
  static constexpr int NT = (kUtRows / 4) * TC;    // threads per CTA
};

inline size_t uvu_tile_smem(int ut, int V, int W2, int np, int n1, int n2) {
  const size_t vc = static_cast<size_t>(V < kUtVC ? V : kUtVC);
  const size_t floats = static_cast<size_t>(W2) * kUtRows + kUtStages * vc * ut +
                        static_cast<size_t>(np) * 8;
  const size_t aligned_floats = (floats + 3) & ~size_t(3);
  const size_t ints = static_cast<size_t>(np) * 4 + static_cast<size_t>(n1 + n2) * 2 + np;
  return 128 + (aligned_floats + ints) * 4;
}

template <class Body>
__device__ __forceinline__ void with_entry_dims(int d1, int d3, Body&& body) {
  if (d1 == 2) {
    if (d3 == 2) body.template operator()<2, 2>(); else body.template operator()<2, 1>();
  } else {
    if (d3 == 2) body.template operator()<1, 2>(); else body.template operator()<1, 1>();
  }
}

template <int D>
__device__ __forceinline__ void ut_load4(float (&v)[4 * D], const float* __restrict__ src,
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
__device__ __forceinline__ void ut_store4(float* __restrict__ dst, const float (&v)[4][2],
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

template <int MODE, int UT, int NH>
__global__ void __launch_bounds__(UtShape<UT, NH>::NT, 1) uvu_tile(UvuTileArgs A) {
  constexpr int TC = UtShape<UT, NH>::TC, NT = UtShape<UT, NH>::NT;
  constexpr int CW = 4 * NH;  // channels per thread
  constexpr int RT = kUtRows;
  extern __shared__ __align__(128) unsigned char ut_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(ut_raw);
  unsigned* done = reinterpret_cast<unsigned*>(ut_raw + 64);
  float* sm = reinterpret_cast<float*>(ut_raw + 128);
  const int tid = threadIdx.x, lane = tid & 31;
  constexpr int nwarps = NT / 32;
  const int vc = A.V < kUtVC ? A.V : kUtVC;
  const int nkc = (A.V + kUtVC - 1) / kUtVC;
  const int np = A.t.np;
  float* Yt = sm;                                          // [W2][RT]
  float* Wt = Yt + static_cast<size_t>(A.W2) * RT;         // [kUtStages][vc][UT]
  float* coef = Wt + kUtStages * vc * UT;                  // [np][8]
  float* fend = coef + np * 8;
  int4* paths = reinterpret_cast<int4*>(sm + ((fend - sm + 3) & ~3));
  int2* in1 = reinterpret_cast<int2*>(paths + np);
  int2* in2 = in1 + A.t.n1;
  int* order = reinterpret_cast<int*>(in2 + A.t.n2);
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * RT;
  const int ub = blockIdx.y * UT;

  for (int q = tid; q < np; q += NT) {
    paths[q] = A.t.paths[q];
    order[q] = MODE == kUtDx ? A.t.by_i[q] : q;
  }
  for (int q = tid; q < np * 8; q += NT) coef[q] = __ldg(A.t.coef + q);
  for (int q = tid; q < A.t.n1; q += NT) in1[q] = A.t.in1[q];
  for (int q = tid; q < A.t.n2; q += NT) in2[q] = A.t.in2[q];
  for (int idx = tid; idx < RT * A.W2; idx += NT) {
    const int r = idx / A.W2, c = idx - r * A.W2;
    const int64_t row = row0 + r;
    Yt[c * RT + r] = row < A.rows ? __ldg(A.y + row * A.W2 + c) : 0.f;
  }
  const int ucopy = A.Up - ub < UT ? A.Up - ub : UT;
  if (ucopy < UT)
    for (int idx = tid; idx < kUtStages * vc * UT; idx += NT) Wt[idx] = 0.f;
  if (tid == 0) {
    for (int st = 0; st < kUtStages; ++st) {
      mbar_init(&full[st], 1);
      done[st] = 0;
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  const int tc = tid % TC, tr = tid / TC;
  const int r0 = tr * 4;
  const int ntiles = np * nkc;
  auto issue = [&](int T, int st) {
    const int p = order[T / nkc], v0 = (T % nkc) * kUtVC;
    const int kn = A.V - v0 < kUtVC ? A.V - v0 : kUtVC;
    float* dst = Wt + st * vc * UT;
    const float* src = A.wt + (static_cast<int64_t>(p) * A.V + v0) * A.Up + ub;
    const uint32_t row_bytes = static_cast<uint32_t>(ucopy) * 4u;
    mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(kn) * row_bytes);
    if (ucopy == UT && A.Up == UT) {
      bulk_g2s(dst, src, static_cast<uint32_t>(kn) * row_bytes, &full[st]);
    } else {
      for (int k = 0; k < kn; ++k) bulk_g2s(dst + k * UT, src + k * A.Up, row_bytes, &full[st]);
    }
  };

  float2 acc[2][4][CW / 2];  // projections, paired along the channels
  float res[4][CW][2];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < CW; ++b) res[a][b][0] = res[a][b][1] = 0.f;

  if (tid == 0)
    for (int T = 0; T < kUtStages && T < ntiles; ++T) issue(T, T);
  bool ok = true;
  // (path position, weight chunk) of tile T, advanced per tile (no division per tile)
  int pos = 0, ck = 0;
  auto advance = [&]() {
    if (++ck == nkc) {
      ck = 0;
      ++pos;
    }
  };
  for (int T = 0; T < ntiles && ok; ++T, advance()) {
    const int st = T % kUtStages;
    const uint32_t round = static_cast<uint32_t>(T / kUtStages);
    ok = mbar_wait(&full[st], round & 1, 7);
    if (!ok) break;
    const int p = order[pos];
    const int4 pt = paths[p];
    const int2 ej = in2[pt.y];
    if (ck == 0) {
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int j = 0; j < CW / 2; ++j) acc[b][a][j] = make_float2(0.f, 0.f);
    }
    const int v0 = ck * kUtVC;
    const int kn = A.V - v0 < kUtVC ? A.V - v0 : kUtVC;
    const float* Wb = Wt + st * vc * UT;
    auto gemm = [&]<int D2>() {
      auto vstep = [&](int v) {
        float2 wv[CW / 2];
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          const float4 w4 = *reinterpret_cast<const float4*>(Wb + v * UT + h * (UT / NH) + tc * 4);
          wv[2 * h] = make_float2(w4.x, w4.y);
          wv[2 * h + 1] = make_float2(w4.z, w4.w);
        }
#pragma unroll
        for (int b = 0; b < D2; ++b) {
          const float4 a4 =
              *reinterpret_cast<const float4*>(Yt + (ej.x + (v0 + v) * D2 + b) * RT + r0);
          const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < CW / 2; ++j) acc[b][i][j] = fma2(av[i], wv[j], acc[b][i][j]);
        }
      };
      // a full chunk fully unrolled (the shared-memory loads of later v issue ahead
      // of the FMAs of earlier ones; 128 registers, no spills); a partial last
      // chunk one v at a time
      if (kn == kUtVC) {
#pragma unroll
        for (int v = 0; v < kUtVC; ++v) vstep(v);
      } else {
        for (int v = 0; v < kn; ++v) vstep(v);
      }
    };
    if (ej.y == 2) gemm.template operator()<2>(); else gemm.template operator()<1>();
    // release the stage; the last warp out refills it
    __syncwarp();
    if (lane == 0) {
      unsigned prev;
      asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                   : "=r"(prev)
                   : "r"(smem_addr(&done[st]))
                   : "memory");
      if (prev + 1 == static_cast<unsigned>(nwarps) * (round + 1)) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (T + kUtStages < ntiles) issue(T + kUtStages, st);
      }
    }
    if (ck != nkc - 1) continue;
    const int2 ei = in1[pt.x], ek = in1[pt.z];
    const float* c = coef + 8 * p;
    const int key = MODE == kUtFwd ? pt.z : pt.x;
    with_entry_dims(ei.y, ek.y, [&]<int D1, int D3>() {
#pragma unroll
      for (int ee = 0; ee < 4; ++ee) {
        const int64_t row = row0 + r0 + ee;
        const bool row_ok = row < A.rows;
#pragma unroll
        for (int half = 0; half < NH; ++half) {
          const int u = ub + half * (UT / NH) + tc * 4;
          if (MODE == kUtFwd) {
            float xv[4 * D1];
            ut_load4<D1>(xv, A.opnd + row * A.W1 + ei.x + static_cast<int64_t>(u) * D1, row_ok,
                         u, A.U, A.vec);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float p0 = pair_at(acc[0][ee], half * 4 + q), p1 = pair_at(acc[1][ee], half * 4 + q);
              const float x0 = xv[q * D1], x1 = D1 == 2 ? xv[q * D1 + 1] : 0.f;
              // out[kc] += sum_{a,b} c[4 kc + 2 a + b] x[a] proj[b]
              float t0 = fmaf(c[1], p1, c[0] * p0);
              if (D1 == 2) t0 = fmaf(x1, fmaf(c[3], p1, c[2] * p0), t0 * x0);
              else t0 = t0 * x0;
              res[ee][half * 4 + q][0] += t0;
              if (D3 == 2) {
                float t1 = fmaf(c[5], p1, c[4] * p0);
                if (D1 == 2) t1 = fmaf(x1, fmaf(c[7], p1, c[6] * p0), t1 * x0);
                else t1 = t1 * x0;
                res[ee][half * 4 + q][1] += t1;
              }
            }
          } else {
            float gv[4 * D3];
            ut_load4<D3>(gv, A.opnd + row * A.W1 + ek.x + static_cast<int64_t>(u) * D3, row_ok,
                         u, A.U, A.vec);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float p0 = pair_at(acc[0][ee], half * 4 + q), p1 = pair_at(acc[1][ee], half * 4 + q);
              const float g0 = gv[q * D3], g1 = D3 == 2 ? gv[q * D3 + 1] : 0.f;
              // dx[a] += sum_{kc,b} c[4 kc + 2 a + b] g[kc] proj[b]
              float s0 = g0 * fmaf(c[1], p1, c[0] * p0);
              if (D3 == 2) s0 = fmaf(g1, fmaf(c[5], p1, c[4] * p0), s0);
              res[ee][half * 4 + q][0] += s0;
              if (D1 == 2) {
                float s1 = g0 * fmaf(c[3], p1, c[2] * p0);
                if (D3 == 2) s1 = fmaf(g1, fmaf(c[7], p1, c[6] * p0), s1);
                res[ee][half * 4 + q][1] += s1;
              }
            }
          }
        }
      }
    });
    const bool last = pos + 1 == np ||
                      (MODE == kUtFwd ? paths[order[pos + 1]].z : paths[order[pos + 1]].x) != key;
    if (last) {
      const int2 eo = in1[key];
#pragma unroll
      for (int ee = 0; ee < 4; ++ee) {
        const int64_t row = row0 + r0 + ee;
        const bool row_ok = row < A.rows;
#pragma unroll
        for (int half = 0; half < NH; ++half) {
          const int u = ub + half * (UT / NH) + tc * 4;
          float vv[4][2];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            vv[q][0] = res[ee][half * 4 + q][0];
            vv[q][1] = res[ee][half * 4 + q][1];
          }
          float* dst = A.out + row * A.W1 + eo.x + static_cast<int64_t>(u) * eo.y;
          if (eo.y == 2) ut_store4<2>(dst, vv, row_ok, u, A.U, A.vec);
          else ut_store4<1>(dst, vv, row_ok, u, A.U, A.vec);
        }
#pragma unroll
        for (int b = 0; b < CW; ++b) res[ee][b][0] = res[ee][b][1] = 0.f;
      }
    }
  }
  if (!ok && tid == 0) {
    // a wait ran out: let copies already issued land before the CTA exits
    for (int st = 0; st < kUtStages; ++st) mbar_wait(&full[st], 0, 8, kDrainLimitNs);
  }
}

template <int MODE, int UT, int NH>
int launch_uvu_tile_shape(const UvuTileArgs& ua, size_t smem, cudaStream_t s) {
  const void* fn = reinterpret_cast<const void*>(&uvu_tile<MODE, UT, NH>);
  const int st = allow_smem(fn, smem);
  if (st != ICTC_OK) return st;
  const dim3 grid(static_cast<unsigned>(ceil_div(ua.rows, kUtRows)),
                  static_cast<unsigned>(ceil_div(ua.U, UT)));
  uvu_tile<MODE, UT, NH><<<grid, UtShape<UT, NH>::NT, smem, s>>>(ua);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "uvu tile launch");
}

// Thread tile of uvu_tile: "wide" (4 x 4 per thread, the default: forward and dx
// -18 % at config 4) or, with ICTC_UVU_TILE=split, 4 x 8; tests cover both.
inline bool uvu_tile_wide() {
  const char* v = getenv("ICTC_UVU_TILE");
  return v == nullptr || strcmp(v, "split") != 0;
}

// Launches uvu_tile<MODE> when its shared-memory tiles fit; returns
// ICTC_ERR_UNSUPPORTED (nothing launched) when they do not.
template <int MODE>
int launch_uvu_tile(const UvuTileArgs& ua, cudaStream_t s) {
  const int ut = ua.U <= 64 ? 64 : 128;
  const size_t smem = uvu_tile_smem(ut, ua.V, ua.W2, ua.t.np, ua.t.n1, ua.t.n2);
  if (smem > 225 * 1024) return ICTC_ERR_UNSUPPORTED;
  const bool wide = uvu_tile_wide();
  if (ut == 64)
    return wide ? launch_uvu_tile_shape<MODE, 64, 1>(ua, smem, s)
                : launch_uvu_tile_shape<MODE, 64, 2>(ua, smem, s);
  return wide ? launch_uvu_tile_shape<MODE, 128, 1>(ua, smem, s)
              : launch_uvu_tile_shape<MODE, 128, 2>(ua, smem, s);
}
