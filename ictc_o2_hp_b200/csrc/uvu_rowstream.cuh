// Per-row-weight uvu forward and VJP: uvu_rowstream<MODE>.
//
// With one weight tensor per row (shared_weights=False) every weight is used by
// exactly one row, so the product is bound by streaming the [rows, P, U, V]
// weights (and, in the VJP, writing as many weight gradients).  A persistent CTA
// per SM takes rows in turn; each row's weights arrive as path chunks of at most
// 4096 floats ([u][v] rows, contiguous in HBM) through a 4-stage ring of bulk
// asynchronous copies, refilled by the last warp that releases a stage, so HBM
// streams continuously across path and row boundaries.
//
// Thread layout per chunk: two threads per channel u (lanes 2u', 2u'+1 split the
// v range); a warp owns 16 consecutive channels of the chunk.  They read the
// chunk's [u][v] rows as float4 in a rotated order ((2s + half + 2u') mod V/4),
// which keeps the eight lanes of each shared-memory phase on distinct banks.
//   forward:  proj[u,b] = sum_v w[u,v] y_j[v,b];  out_k[u] += c x_i proj
//   VJP:      proj as above, dx_i[u] += c g_k proj;
//             s[u,b] = sum c[kc][a][b] g_k[u,kc] x_i[u,a];
//             dw[u,v] = sum_b s[u,b] y_j[v,b]   (coalesced float4 stores per warp)
//             dy_j[v,b] += sum_u w[u,v] s[u,b] (lane v, per-warp partial rows)
// The slot vectors of x, g and the output / dx accumulators live in shared
// memory as [2 n1][U]; per-warp dy partials are summed in warp order per row.
//
// This header is included inside the anonymous namespace of uvu_kernels.cu.
#pragma once

enum RowStreamMode { kRsFwd = 0, kRsBwd = 1 };
constexpr int kRsThreads = 256;
constexpr int kRsStages = 4;
constexpr int kRsChunk = 4096;  // floats per ring stage

struct RowStreamArgs {
  const float* x; const float* y; const float* w; const float* g;
  float* out;   // forward output, or dx
  float* dy; float* dw;
  int64_t rows, Wn;
  int U, V, W1, W2;
  UvuDev t;
  int needed;   // VJP roles: 1 dx, 2 dy, 4 dw
};

// Channels per ring chunk: whole [u][v] rows, at most kRsChunk floats and 128
// channels (two threads per channel).
__host__ __device__ inline int rowstream_chunk_u(int U, int V) {
  int cu = kRsChunk / V;
  if (cu > 128) cu = 128;
  if (cu > U) cu = U;
  return cu < 1 ? 1 : cu;
}

inline bool rowstream_fits(int U, int V, int W1, int W2, int n1) {
  (void)W1;
  // float4 runs of y_j: V a multiple of 8 keeps every entry offset 16-byte aligned
  if (V % 8 != 0 || V > kRsChunk) return false;
  const size_t smem = 128 + (static_cast<size_t>(kRsStages) * kRsChunk + ((W2 + 3) & ~3) +
                             6 * static_cast<size_t>(n1) * U + 2 * 128 +
                             8 * static_cast<size_t>((W2 + 3) & ~3)) * 4;
  return smem <= 220 * 1024;
}

inline size_t rowstream_smem(int U, int W2, int n1) {
  return 128 + (static_cast<size_t>(kRsStages) * kRsChunk + ((W2 + 3) & ~3) +
                6 * static_cast<size_t>(n1) * U + 2 * 128 +
                8 * static_cast<size_t>((W2 + 3) & ~3)) * 4;
}

template <int MODE>
__global__ void __launch_bounds__(kRsThreads, 2) uvu_rowstream(RowStreamArgs A) {
  extern __shared__ __align__(128) unsigned char rs_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(rs_raw);
  unsigned* done = reinterpret_cast<unsigned*>(rs_raw + 64);
  float* ring = reinterpret_cast<float*>(rs_raw + 128);     // [kRsStages][kRsChunk]
  const int W2a = (A.W2 + 3) & ~3;
  const int n1 = A.t.n1;
  float* ys = ring + kRsStages * kRsChunk;                   // [W2a]
  float* xs = ys + W2a;                                      // [2 n1][U] x slots
  float* gs = xs + 2 * n1 * A.U;                             // [2 n1][U] g slots (VJP)
  float* os = gs + 2 * n1 * A.U;                             // [2 n1][U] out / dx
  float* sb = os + 2 * n1 * A.U;                             // [128][2] s (VJP)
  float* yp = sb + 2 * 128;                                  // [8 warps][W2a] dy partials
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int nwarps = kRsThreads / 32;
  const int cu = rowstream_chunk_u(A.U, A.V);
  const int nch = (A.U + cu - 1) / cu;
  const int per_row = A.t.np * nch;
  const int nv4 = A.V / 4;
  const bool want_dx = MODE == kRsBwd && (A.needed & 1);
  const bool want_dy = MODE == kRsBwd && (A.needed & 2);
  const bool want_dw = MODE == kRsBwd && (A.needed & 4);
  // rows of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int64_t my_rows = A.rows > blockIdx.x ? (A.rows - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t nitems = my_rows * per_row;
  auto issue = [&](int64_t it, int st) {
    const int64_t rl = it / per_row;
    const int rem = static_cast<int>(it - rl * per_row);
    const int p = rem / nch, c = rem - p * nch;
    const int64_t row = blockIdx.x + rl * gridDim.x;
    const int u0 = c * cu;
    const int ncu = A.U - u0 < cu ? A.U - u0 : cu;
    const uint32_t bytes = static_cast<uint32_t>(ncu) * A.V * 4u;
    mbar_arrive_expect_tx(&full[st], bytes);
    bulk_g2s(ring + st * kRsChunk, A.w + row * A.Wn + (static_cast<int64_t>(p) * A.U + u0) * A.V,
             bytes, &full[st]);
  };
  if (tid == 0) {
    for (int st = 0; st < kRsStages; ++st) {
      mbar_init(&full[st], 1);
      done[st] = 0;
    }
    fence_mbarrier_init();
    for (int st = 0; st < kRsStages && st < nitems; ++st) issue(st, st);
  }
  const int ul = (tid & 31) >> 1;    // channel within the warp's 16
  const int half = tid & 1;
  bool ok = true;
  int64_t it = 0;
  for (int64_t rl = 0; rl < my_rows && ok; ++rl) {
    const int64_t row = blockIdx.x + rl * gridDim.x;
    __syncthreads();  // previous row's outputs are written
    for (int q = tid; q < A.W2; q += kRsThreads) ys[q] = __ldg(A.y + row * A.W2 + q);
    for (int q = tid; q < 2 * n1 * A.U; q += kRsThreads) {
      const int e = q / (2 * A.U), r = q - e * 2 * A.U;
      const int comp = r / A.U, u = r - comp * A.U;
      const int2 en = A.t.in1[e];
      const int64_t o = row * A.W1 + en.x + static_cast<int64_t>(u) * en.y + comp;
      const bool has = comp < en.y;
      xs[q] = (MODE == kRsFwd || want_dy || want_dw) && has ? __ldg(A.x + o) : 0.f;
      if (MODE == kRsBwd) gs[q] = has ? __ldg(A.g + o) : 0.f;
      os[q] = 0.f;
    }
    if (want_dy)
      for (int q = tid; q < nwarps * W2a; q += kRsThreads) yp[q] = 0.f;
    __syncthreads();
    for (int item = 0; item < per_row; ++item, ++it) {
      const int st = static_cast<int>(it % kRsStages);
      const uint32_t round = static_cast<uint32_t>(it / kRsStages);
      ok = mbar_wait(&full[st], round & 1, 9);
      if (!ok) break;
      const int p = item / nch, c = item - p * nch;
      const int u0 = c * cu;
      const int ncu = A.U - u0 < cu ? A.U - u0 : cu;
      const int4 pt = A.t.paths[p];
      const int2 ej = A.t.in2[pt.y];
      const float* cf = A.t.coef + 8 * p;
      const float* wc = ring + st * kRsChunk;
      const int uw = warp * 16 + ul;        // channel within the chunk
      const bool act = uw < ncu;
      const int u = u0 + uw;
      // y_j as float4 runs: entry offsets are multiples of V (a multiple of 8)
      auto body = [&]<int D2>() {
        const float* yj = ys + ej.x;
        // proj[b] over this thread's half of v, rotated float4 order, two chains
        float pa0 = 0.f, pa1 = 0.f, pb0 = 0.f, pb1 = 0.f;
        if (act) {
          int f = half + 2 * ul;
          f = f % nv4;
          for (int s2 = 0; s2 < nv4; s2 += 2) {
            const float4 w4 = *reinterpret_cast<const float4*>(wc + uw * A.V + f * 4);
            if (D2 == 2) {
              const float4 y0 = *reinterpret_cast<const float4*>(yj + f * 8);
              const float4 y1 = *reinterpret_cast<const float4*>(yj + f * 8 + 4);
              pa0 = fmaf(w4.x, y0.x, pa0); pa1 = fmaf(w4.x, y0.y, pa1);
              pb0 = fmaf(w4.y, y0.z, pb0); pb1 = fmaf(w4.y, y0.w, pb1);
              pa0 = fmaf(w4.z, y1.x, pa0); pa1 = fmaf(w4.z, y1.y, pa1);
              pb0 = fmaf(w4.w, y1.z, pb0); pb1 = fmaf(w4.w, y1.w, pb1);
            } else {
              const float4 y0 = *reinterpret_cast<const float4*>(yj + f * 4);
              pa0 = fmaf(w4.x, y0.x, pa0); pb0 = fmaf(w4.y, y0.y, pb0);
              pa0 = fmaf(w4.z, y0.z, pa0); pb0 = fmaf(w4.w, y0.w, pb0);
            }
            f += 2;
            if (f >= nv4) f -= nv4;
          }
        }
        float p0 = pa0 + pb0, p1 = pa1 + pb1;
        p0 += __shfl_xor_sync(0xffffffffu, p0, 1);
        p1 += __shfl_xor_sync(0xffffffffu, p1, 1);
        float s0 = 0.f, s1 = 0.f;
        if (act) {
          const float c0 = __ldg(cf), c1 = __ldg(cf + 1), c2 = __ldg(cf + 2), c3 = __ldg(cf + 3);
          const float c4 = __ldg(cf + 4), c5 = __ldg(cf + 5), c6 = __ldg(cf + 6), c7 = __ldg(cf + 7);
          const float x0 = xs[(2 * pt.x) * A.U + u], x1 = xs[(2 * pt.x + 1) * A.U + u];
          if (MODE == kRsFwd) {
            if (half == 0) {
              os[(2 * pt.z) * A.U + u] += x0 * fmaf(c1, p1, c0 * p0) + x1 * fmaf(c3, p1, c2 * p0);
              os[(2 * pt.z + 1) * A.U + u] +=
                  x0 * fmaf(c5, p1, c4 * p0) + x1 * fmaf(c7, p1, c6 * p0);
            }
          } else {
            const float g0 = gs[(2 * pt.z) * A.U + u], g1 = gs[(2 * pt.z + 1) * A.U + u];
            if (want_dx && half == 0) {
              os[(2 * pt.x) * A.U + u] += g0 * fmaf(c1, p1, c0 * p0) + g1 * fmaf(c5, p1, c4 * p0);
              os[(2 * pt.x + 1) * A.U + u] +=
                  g0 * fmaf(c3, p1, c2 * p0) + g1 * fmaf(c7, p1, c6 * p0);
            }
            // s[b] = sum_{kc,a} c[4 kc + 2 a + b] g[kc] x[a]
            s0 = g0 * fmaf(c2, x1, c0 * x0) + g1 * fmaf(c6, x1, c4 * x0);
            s1 = g0 * fmaf(c3, x1, c1 * x0) + g1 * fmaf(c7, x1, c5 * x0);
          }
        }
        if (MODE == kRsBwd && (want_dw || want_dy)) {
          float* swarp = sb + warp * 32;  // [16 channels][2] of this warp
          if (half == 0) {
            swarp[2 * ul] = s0;
            swarp[2 * ul + 1] = s1;
          }
          __syncwarp();
          const int nu = ncu - warp * 16 < 16 ? ncu - warp * 16 : 16;
          if (want_dw && nu > 0) {
            float* dst = A.dw + row * A.Wn + (static_cast<int64_t>(p) * A.U + u0 + warp * 16) * A.V;
            for (int q = lane; q < nu * nv4; q += 32) {
              const int uu = q / nv4, fq = q - uu * nv4;
              const float a0 = swarp[2 * uu], a1 = swarp[2 * uu + 1];
              float4 o;
              if (D2 == 2) {
                const float4 y0 = *reinterpret_cast<const float4*>(yj + fq * 8);
                const float4 y1 = *reinterpret_cast<const float4*>(yj + fq * 8 + 4);
                o.x = fmaf(a1, y0.y, a0 * y0.x);
                o.y = fmaf(a1, y0.w, a0 * y0.z);
                o.z = fmaf(a1, y1.y, a0 * y1.x);
                o.w = fmaf(a1, y1.w, a0 * y1.z);
              } else {
                const float4 y0 = *reinterpret_cast<const float4*>(yj + fq * 4);
                o = make_float4(a0 * y0.x, a0 * y0.y, a0 * y0.z, a0 * y0.w);
              }
              reinterpret_cast<float4*>(dst + uu * A.V)[fq] = o;
            }
          }
          if (want_dy && nu > 0) {
            for (int v = lane; v < A.V; v += 32) {
              float d0a = 0.f, d1a = 0.f, d0b = 0.f, d1b = 0.f;
              const float* wcol = wc + (warp * 16) * A.V + v;
              int uu = 0;
              for (; uu + 1 < nu; uu += 2) {
                const float w0 = wcol[uu * A.V], w1 = wcol[(uu + 1) * A.V];
                d0a = fmaf(w0, swarp[2 * uu], d0a);
                d1a = fmaf(w0, swarp[2 * uu + 1], d1a);
                d0b = fmaf(w1, swarp[2 * uu + 2], d0b);
                d1b = fmaf(w1, swarp[2 * uu + 3], d1b);
              }
              if (uu < nu) {
                const float w0 = wcol[uu * A.V];
                d0a = fmaf(w0, swarp[2 * uu], d0a);
                d1a = fmaf(w0, swarp[2 * uu + 1], d1a);
              }
              yp[warp * W2a + ej.x + v * D2] += d0a + d0b;
              if (D2 == 2) yp[warp * W2a + ej.x + v * 2 + 1] += d1a + d1b;
            }
          }
          __syncwarp();
        }
      };
      if (ej.y == 2) body.template operator()<2>(); else body.template operator()<1>();
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
          if (it + kRsStages < nitems) issue(it + kRsStages, st);
        }
      }
    }
    // one verdict for the whole CTA, so every thread takes the same barriers
    if (!__syncthreads_and(ok)) {
      ok = false;
      break;
    }
    if (MODE == kRsFwd || want_dx) {
      for (int q = tid; q < 2 * n1 * A.U; q += kRsThreads) {
        const int e = q / (2 * A.U), r = q - e * 2 * A.U;
        const int comp = r / A.U, u = r - comp * A.U;
        const int2 en = A.t.in1[e];
        if (comp < en.y) A.out[row * A.W1 + en.x + static_cast<int64_t>(u) * en.y + comp] = os[q];
      }
    }
    if (want_dy) {
      for (int q = tid; q < A.W2; q += kRsThreads) {
        float sum = 0.f;
        for (int k = 0; k < nwarps; ++k) sum += yp[k * W2a + q];
        A.dy[row * A.W2 + q] = sum;
      }
    }
  }
  if (!ok && tid == 0) {
    // a wait ran out: let copies already issued land before the CTA exits
    for (int st = 0; st < kRsStages; ++st) mbar_wait(&full[st], 0, 10, kDrainLimitNs);
  }
}
