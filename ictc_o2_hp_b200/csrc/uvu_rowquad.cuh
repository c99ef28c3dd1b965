// Per-row-weight uvu forward and VJP for V in {8, 16, 32, 64}: uvu_rowquad<MODE, NQ, R>.
//
// Same stream as uvu_rowstream (persistent CTAs take rows in turn; each row's
// [P][U][V] weights arrive as chunks of whole [u][v] rows through a ring of bulk
// asynchronous copies (4 stages), refilled by the last warp that releases a
// stage),
// with a thread layout that keeps every operand but the weights in registers:
//
//   * a lane owns one float4 column q of V (QT columns when V = 64) of R channel
//     rows of the chunk (rows group * R + r when a row spans 8 lanes, else
//     r * G + group, G channel-row groups per CTA).  Each 8-lane phase of a warp
//     read covers 128 contiguous bytes of the stage (no bank conflicts without
//     any rotation), the rows owned after the proj reduction are consecutive
//     channels (conflict-free slot accesses), and the lane releases the stage as
//     soon as its R x QT float4 are in registers;
//   * y_j[v, b] of the lane's columns sits in registers for the path;
//   * proj[u, b] = sum_v w[u, v] y_j[v, b] is reduced over the L lanes of a row
//     group by a reduce-scatter (each lane ends with one channel row);
//   * VJP: s[u, b] = sum c[kc][a][b] g_k[u, kc] x_i[u, a] is formed by the lane
//     that owns row u and gathered by shuffles; dw[u, v] = sum_b s y_j is stored
//     as coalesced float4 rows; dy_j[v, b] = sum_u w s is reduced over the
//     warp's row groups by another reduce-scatter and added to a per-warp
//     partial row, summed over the warps in a fixed order per row.
//
// Template parameters: NQ = V / 4 float4 columns per channel row, R channel rows
// per lane (R <= lanes per row, R x QT <= 4 so a chunk fits one ring stage).
//
// This header is included inside the anonymous namespace of uvu_kernels.cu,
// after uvu_rowstream.cuh (RowStreamArgs, kRsChunk, kRsThreads).
#pragma once

template <int NQ>
struct RqShape {
  static constexpr int L = NQ < 8 ? NQ : 8;  // lanes per channel row
  static constexpr int QT = NQ / L;          // float4 columns per lane
  static constexpr int GW = 32 / L;          // channel-row groups per warp
  static constexpr int G = 8 * GW;           // channel-row groups per CTA (8 warps)
  // chunk row of (group, r): group-major when a row spans 8 lanes (one 8-lane
  // phase per row either way; consecutive channels for the row owners)
  static constexpr bool kGroupMajor = L == 8;
  template <int R>
  __device__ __forceinline__ static int row(int group, int r) {
    return kGroupMajor ? group * R + r : r * G + group;
  }
};

// Ring depth (a fifth forward stage, which fits at two CTAs per SM, measured no
// faster).
template <int MODE>
constexpr int rq_stages() { return 4; }

// Shared memory of uvu_rowquad: barriers, ring, y, x (/ g) / out slots, per-warp
// dy partials (VJP), per-path records.
template <int MODE>
inline size_t rowquad_smem(int U, int W2, int n1, int np) {
  const size_t w2a = static_cast<size_t>((W2 + 3) & ~3);
  const size_t slots = (MODE == kRsFwd ? 4 : 6) * static_cast<size_t>(n1) * U;
  const size_t before = static_cast<size_t>(rq_stages<MODE>()) * kRsChunk + w2a + slots +
                        (MODE == kRsFwd ? 0 : 8 * w2a);
  return 128 + (((before + 3) & ~size_t(3)) + 4 * static_cast<size_t>(np)) * 4;
}

// Reduce-scatter of v over the lanes lane ^ m for m = M, M / 2, ..., S: while more
// than MINB values remain, each level keeps one half (the upper half on lanes
// with bit m set) and adds the partner's copy of it; later levels sum all
// remaining values.  On return v[0 .. CNT) holds the lane's block in order.
template <int NV, int CNT, int M, int S, int MINB>
__device__ __forceinline__ void rq_reduce(float (&v)[NV], int lane) {
  if constexpr (M >= S) {
    if constexpr (CNT > MINB) {
      constexpr int H = CNT / 2;
      const bool upper = (lane & M) != 0;
#pragma unroll
      for (int k = 0; k < H; ++k) {
        const float send = upper ? v[k] : v[k + H];
        const float keep = upper ? v[k + H] : v[k];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, M);
      }
      rq_reduce<NV, H, M / 2, S, MINB>(v, lane);
    } else {
#pragma unroll
      for (int k = 0; k < CNT; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], M);
      rq_reduce<NV, CNT, M / 2, S, MINB>(v, lane);
    }
  }
}

// First value index of the block rq_reduce leaves on `lane`.
template <int CNT, int M, int S, int MINB>
__device__ __forceinline__ int rq_block(int lane) {
  if constexpr (M >= S && CNT > MINB)
    return ((lane & M) ? CNT / 2 : 0) + rq_block<CNT / 2, M / 2, S, MINB>(lane);
  else
    return 0;
}

// Lane bits of the levels that only summed (lanes differing there hold equal blocks).
template <int CNT, int M, int S, int MINB>
constexpr int rq_redundant() {
  if constexpr (M < S)
    return 0;
  else if constexpr (CNT > MINB)
    return rq_redundant<CNT / 2, M / 2, S, MINB>();
  else
    return M | rq_redundant<CNT, M / 2, S, MINB>();
}

// Number of float4 per 8-float run of y_j loaded for one column (D2 values per v).
template <int D2>
__device__ __forceinline__ void rq_load_y(float (&yv)[4][2], const float* src) {
  if constexpr (D2 == 2) {
    const float4 a = *reinterpret_cast<const float4*>(src);
    const float4 b = *reinterpret_cast<const float4*>(src + 4);
    yv[0][0] = a.x; yv[0][1] = a.y; yv[1][0] = a.z; yv[1][1] = a.w;
    yv[2][0] = b.x; yv[2][1] = b.y; yv[3][0] = b.z; yv[3][1] = b.w;
  } else {
    const float4 a = *reinterpret_cast<const float4*>(src);
    yv[0][0] = a.x; yv[1][0] = a.y; yv[2][0] = a.z; yv[3][0] = a.w;
    yv[0][1] = yv[1][1] = yv[2][1] = yv[3][1] = 0.f;
  }
}

__device__ __forceinline__ float rq_get(const float4& a, int e) {
  return e == 0 ? a.x : (e == 1 ? a.y : (e == 2 ? a.z : a.w));
}

template <int MODE, int NQ, int R>
__global__ void __launch_bounds__(kRsThreads, 2) uvu_rowquad(RowStreamArgs A) {
  using Sh = RqShape<NQ>;
  constexpr int L = Sh::L, QT = Sh::QT, GW = Sh::GW, G = Sh::G;
  constexpr int V = 4 * NQ;
  constexpr int CU = G * R;  // channel rows per chunk
  constexpr int NS = rq_stages<MODE>();
  static_assert(R <= L && R * QT <= 4 && CU * V <= kRsChunk, "chunk shape");
  extern __shared__ __align__(128) unsigned char rq_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(rq_raw);
  unsigned* done = reinterpret_cast<unsigned*>(rq_raw + 64);
  float* ring = reinterpret_cast<float*>(rq_raw + 128);  // [NS][kRsChunk]
  const int W2a = (A.W2 + 3) & ~3;
  const int n1 = A.t.n1, np = A.t.np, U = A.U;
  float* ys = ring + NS * kRsChunk;  // [W2a]
  float* xs = ys + W2a;              // [2 n1][U] x slots
  float* gs = xs + 2 * n1 * U;       // [2 n1][U] g slots (VJP only)
  float* os = gs + (MODE == kRsBwd ? 2 * n1 * U : 0);  // [2 n1][U] out / dx
  float* yp = os + 2 * n1 * U;       // [8 warps][W2a] dy partials (VJP only)
  // per path: x slot offset, out / g slot offset, y_j offset, y_j dim (16-byte aligned)
  int4* meta = reinterpret_cast<int4*>(
      ring + ((static_cast<int>(yp - ring) + (MODE == kRsBwd ? 8 * W2a : 0) + 3) & ~3));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ql = lane % L;
  const int grp = warp * GW + lane / L;
  const int nch = (U + CU - 1) / CU;
  const int per_row = np * nch;
  const bool want_dx = MODE == kRsBwd && (A.needed & 1);
  const bool want_dy = MODE == kRsBwd && (A.needed & 2);
  const bool want_dw = MODE == kRsBwd && (A.needed & 4);
  // the channel row a lane owns after the proj reduction, and whether it writes
  const int rl = ql / (L / R);
  const bool leader = (ql % (L / R)) == 0;
  const int own = Sh::template row<R>(grp, rl);  // chunk row this lane owns
  for (int q = tid; q < np; q += kRsThreads) {
    const int4 pt = __ldg(A.t.paths + q);
    const int2 ej = __ldg(A.t.in2 + pt.y);
    meta[q] = make_int4(2 * pt.x * U, 2 * pt.z * U, ej.x, ej.y);
  }
  const int64_t my_rows = A.rows > blockIdx.x ? (A.rows - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t nitems = my_rows * per_row;
  // item -> (row, chunk c, path p), chunk-major within a row
  auto issue = [&](int64_t item_id, int st) {
    const int64_t r_local = item_id / per_row;
    const int rem = static_cast<int>(item_id - r_local * per_row);
    const int c = rem / np, p = rem - c * np;
    const int64_t row = blockIdx.x + r_local * gridDim.x;
    const int u0 = c * CU;
    const int ncu = U - u0 < CU ? U - u0 : CU;
    const uint32_t bytes = static_cast<uint32_t>(ncu) * V * 4u;
    mbar_arrive_expect_tx(&full[st], bytes);
    bulk_g2s(ring + st * kRsChunk, A.w + row * A.Wn + (static_cast<int64_t>(p) * U + u0) * V,
             bytes, &full[st]);
  };
  if (tid == 0) {
    for (int st = 0; st < NS; ++st) {
      mbar_init(&full[st], 1);
      done[st] = 0;
    }
    fence_mbarrier_init();
    for (int st = 0; st < NS && st < nitems; ++st) issue(st, st);
  }
  bool ok = true;
  int64_t it = 0;
  for (int64_t r_local = 0; r_local < my_rows && ok; ++r_local) {
    const int64_t row = blockIdx.x + r_local * gridDim.x;
    __syncthreads();  // previous row's outputs are written
    for (int q = tid; q < A.W2; q += kRsThreads) ys[q] = __ldg(A.y + row * A.W2 + q);
    for (int q = tid; q < 2 * n1 * U; q += kRsThreads) {
      const int e = q / (2 * U), r = q - e * 2 * U;
      const int comp = r / U, u = r - comp * U;
      const int2 en = A.t.in1[e];
      const int64_t o = row * A.W1 + en.x + static_cast<int64_t>(u) * en.y + comp;
      const bool has = comp < en.y;
      xs[q] = (MODE == kRsFwd || want_dy || want_dw) && has ? __ldg(A.x + o) : 0.f;
      if (MODE == kRsBwd) gs[q] = has ? __ldg(A.g + o) : 0.f;
      os[q] = 0.f;
    }
    if (want_dy)
      for (int q = tid; q < 8 * W2a; q += kRsThreads) yp[q] = 0.f;
    __syncthreads();
    int c = 0, p = 0;
    for (int item = 0; item < per_row; ++item, ++it) {
      const int st = static_cast<int>(it % NS);
      // c[kc * 4 + a * 2 + b]; in flight while the stage lands
      const float4 ca = __ldg(reinterpret_cast<const float4*>(A.t.coef + 8 * p));
      const float4 cb = __ldg(reinterpret_cast<const float4*>(A.t.coef + 8 * p + 4));
      ok = mbar_wait(&full[st], static_cast<uint32_t>(it / NS) & 1u, 11);
      if (!ok) break;
      const int u0 = c * CU;
      const int ncu = U - u0 < CU ? U - u0 : CU;
      const float* wc = ring + st * kRsChunk;
      float4 w[R][QT];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int uu = Sh::template row<R>(grp, r);
#pragma unroll
        for (int t = 0; t < QT; ++t)
          w[r][t] = uu < ncu ? *reinterpret_cast<const float4*>(wc + uu * V + (ql + L * t) * 4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      // the stage is in registers: release it; the last warp out refills it
      __syncwarp();
      if (lane == 0) {
        unsigned prev;
        asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "r"(smem_addr(&done[st]))
                     : "memory");
        if (prev + 1 == 8u * static_cast<unsigned>(it / NS + 1)) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          if (it + NS < nitems) issue(it + NS, st);
        }
      }
      const int4 pm = meta[p];
      const int xo = pm.x, zo = pm.y;  // slot offsets of x_i and of out_k / g_k
      const int2 ej = make_int2(pm.z, pm.w);
      const float c0 = ca.x, c1 = ca.y, c2 = ca.z, c3 = ca.w;
      const float c4 = cb.x, c5 = cb.y, c6 = cb.z, c7 = cb.w;
      const int uown = u0 + own;  // channel of the row this lane owns
      const bool own_ok = own < ncu;
      auto body = [&]<int D2>() {
        float yv[QT][4][2];
#pragma unroll
        for (int t = 0; t < QT; ++t) rq_load_y<D2>(yv[t], ys + ej.x + (ql + L * t) * 4 * D2);
        if (MODE == kRsFwd || want_dx) {
          float pv[2 * R];
#pragma unroll
          for (int r = 0; r < R; ++r) {
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int t = 0; t < QT; ++t)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float wv = rq_get(w[r][t], e);
                a0 = fmaf(wv, yv[t][e][0], a0);
                if (D2 == 2) a1 = fmaf(wv, yv[t][e][1], a1);
              }
            pv[2 * r] = a0;
            pv[2 * r + 1] = a1;
          }
          rq_reduce<2 * R, 2 * R, L / 2, 1, 2>(pv, lane);
          const float p0 = pv[0], p1 = pv[1];
          if (leader && own_ok) {
            if (MODE == kRsFwd) {
              const float x0 = xs[xo + uown], x1 = xs[xo + U + uown];
              os[zo + uown] += x0 * fmaf(c1, p1, c0 * p0) + x1 * fmaf(c3, p1, c2 * p0);
              os[zo + U + uown] += x0 * fmaf(c5, p1, c4 * p0) + x1 * fmaf(c7, p1, c6 * p0);
            } else {
              const float g0 = gs[zo + uown], g1 = gs[zo + U + uown];
              os[xo + uown] += g0 * fmaf(c1, p1, c0 * p0) + g1 * fmaf(c5, p1, c4 * p0);
              os[xo + U + uown] += g0 * fmaf(c3, p1, c2 * p0) + g1 * fmaf(c7, p1, c6 * p0);
            }
          }
        }
        if (MODE == kRsBwd && (want_dw || want_dy)) {
          // s of the owned row, then gathered for the lane's R rows
          float s0 = 0.f, s1 = 0.f;
          if (own_ok) {
            const float x0 = xs[xo + uown], x1 = xs[xo + U + uown];
            const float g0 = gs[zo + uown], g1 = gs[zo + U + uown];
            s0 = g0 * fmaf(c2, x1, c0 * x0) + g1 * fmaf(c6, x1, c4 * x0);
            s1 = g0 * fmaf(c3, x1, c1 * x0) + g1 * fmaf(c7, x1, c5 * x0);
          }
          float sr[R][2];
          const int gbase = lane - ql;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            sr[r][0] = __shfl_sync(0xffffffffu, s0, gbase + r * (L / R));
            sr[r][1] = __shfl_sync(0xffffffffu, s1, gbase + r * (L / R));
          }
          if (want_dw) {
            float* dst = A.dw + row * A.Wn + (static_cast<int64_t>(p) * U + u0) * V;
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const int uu = Sh::template row<R>(grp, r);
              if (uu < ncu) {
#pragma unroll
                for (int t = 0; t < QT; ++t) {
                  float o[4];
#pragma unroll
                  for (int e = 0; e < 4; ++e)
                    o[e] = D2 == 2 ? fmaf(sr[r][1], yv[t][e][1], sr[r][0] * yv[t][e][0])
                                   : sr[r][0] * yv[t][e][0];
                  *reinterpret_cast<float4*>(dst + uu * V + (ql + L * t) * 4) =
                      make_float4(o[0], o[1], o[2], o[3]);
                }
              }
            }
          }
          if (want_dy) {
            constexpr int NV = QT * 4 * D2;
            float dv[NV];
#pragma unroll
            for (int t = 0; t < QT; ++t)
#pragma unroll
              for (int e = 0; e < 4; ++e)
#pragma unroll
                for (int b = 0; b < D2; ++b) {
                  float a = 0.f;
#pragma unroll
                  for (int r = 0; r < R; ++r) a = fmaf(rq_get(w[r][t], e), sr[r][b], a);
                  dv[(t * 4 + e) * D2 + b] = a;
                }
            rq_reduce<NV, NV, 16, L, 1>(dv, lane);
            constexpr int CNT = NV / GW > 0 ? NV / GW : 1;
            if ((lane & rq_redundant<NV, 16, L, 1>()) == 0) {
              const int n0 = rq_block<NV, 16, L, 1>(lane);
              float* dst = yp + warp * W2a + ej.x;
#pragma unroll
              for (int k = 0; k < CNT; ++k) {
                const int n = n0 + k;
                const int t = n / (4 * D2), e = (n / D2) & 3, b = n % D2;
                dst[((ql + L * t) * 4 + e) * D2 + b] += dv[k];
              }
            }
          }
        }
      };
      if (ej.y == 2) body.template operator()<2>(); else body.template operator()<1>();
      if (++p == np) {
        p = 0;
        ++c;
      }
    }
    // one verdict for the whole CTA, so every thread takes the same barriers
    if (!__syncthreads_and(ok)) {
      ok = false;
      break;
    }
    if (MODE == kRsFwd || want_dx) {
      for (int q = tid; q < 2 * n1 * U; q += kRsThreads) {
        const int e = q / (2 * U), r = q - e * 2 * U;
        const int comp = r / U, u = r - comp * U;
        const int2 en = A.t.in1[e];
        if (comp < en.y) A.out[row * A.W1 + en.x + static_cast<int64_t>(u) * en.y + comp] = os[q];
      }
    }
    if (want_dy) {
      for (int q = tid; q < A.W2; q += kRsThreads) {
        float sum = 0.f;
        for (int k = 0; k < 8; ++k) sum += yp[k * W2a + q];
        A.dy[row * A.W2 + q] = sum;
      }
    }
  }
  if (!ok && tid == 0) {
    // a wait ran out: let copies already issued land before the CTA exits
    for (int st = 0; st < NS; ++st) mbar_wait(&full[st], 0, 12, kDrainLimitNs);
  }
}

// Channel rows per lane for a channel count: the fewest (1, 2, 4) whose chunk
// covers U, within the shape limits.
template <int NQ>
inline int rowquad_rows_per_lane(int U) {
  using Sh = RqShape<NQ>;
  const int rmax = Sh::L < 4 / Sh::QT ? Sh::L : 4 / Sh::QT;
  int r = 1;
  while (r < rmax && Sh::G * r < U) r *= 2;
  return r;
}
