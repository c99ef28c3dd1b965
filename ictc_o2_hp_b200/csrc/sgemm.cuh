// FP32 SIMT GEMM tile for the radial weight gradients: C = A * B, strict FP32.
//
//   A_KMAJOR = false: A is [M][K] row-major (lda = row stride)
//   A_KMAJOR = true:  A is [K][M] row-major (lda = row stride)
//   B is [K][N] row-major (ldb = row stride), N <= 64 per CTA column tile
//
// CTA tile 128 x 64, K steps of 16, 128 threads with 8 x 8 thread tiles split
// in 4 x 4 quarters (rows tm*4.. and 64 + tm*4.., columns tn*4.. and 32 + tn*4..)
// read from k-major shared tiles as float4.  The next K step is fetched into
// registers (A, [M][K] layout: transposed on the way into shared memory) or by
// cp.async (k-major A and B) while the current one is multiplied; one barrier
// per step.  blockIdx.z selects a K chunk [z * k_chunk, ...) whose product is
// written to C + z * c_chunk_stride (callers sum chunks in a fixed order).
//
// Requirements (checked by the callers): K-major rows and B rows 16-byte
// aligned with lda, ldb multiples of 4.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace ictc {

constexpr int kGemmBM = 128, kGemmBN = 64, kGemmBK = 16, kGemmThreads = 128;

struct SgemmArgs {
  const float* A; const float* B; float* C;
  int64_t M, N, K;
  int64_t lda, ldb, ldc;
  int64_t k_chunk;          // K range per blockIdx.z
  int64_t c_chunk_stride;   // floats between the C outputs of consecutive chunks
};

__device__ __forceinline__ void sg_cp16(void* smem, const void* gmem, bool valid) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}

// The accumulators are float2 pairs along the columns (paired f32x2 FMAs, half the
// issue slots of scalar FMAs, bit-identical results).  Register pairs cost the
// [M][K] variant its fit in 128 registers next to the register-staged A rows, so
// it runs 3 CTAs per SM (166 registers) instead of 4 with spills.
template <bool A_KMAJOR>
__global__ void __launch_bounds__(kGemmThreads, A_KMAJOR ? 4 : 3) sgemm_tile(SgemmArgs G) {
  __shared__ __align__(16) float As[2][kGemmBK][kGemmBM];
  __shared__ __align__(16) float Bs[2][kGemmBK][kGemmBN];
  const int tid = threadIdx.x;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kGemmBM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * kGemmBN;
  const int64_t kbeg = static_cast<int64_t>(blockIdx.z) * G.k_chunk;
  const int64_t kend = kbeg + G.k_chunk < G.K ? kbeg + G.k_chunk : G.K;
  const int64_t nsteps = kend > kbeg ? (kend - kbeg + kGemmBK - 1) / kGemmBK : 0;
  const int tm = tid >> 3, tn = tid & 7;

  // A in [M][K]: each thread loads 4 float4 (rows ar + 32 i, k quad ak) into registers
  const int ar = tid >> 2, ak = (tid & 3) * 4;
  float4 areg[4];
  auto load_a_rows = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + ar + 32 * i;
      const int64_t k = k0 + ak;
      if (m < G.M && k + 3 < kend) {
        areg[i] = __ldg(reinterpret_cast<const float4*>(G.A + m * G.lda + k));
      } else {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = (m < G.M && k + j < kend) ? __ldg(G.A + m * G.lda + k + j) : 0.f;
        areg[i] = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
  };
  // Transposed into As[k][m ^ swz(k)]: swz(k) = 8 ((k / 4) % 4) puts the four lanes
  // that share a row m (k quads 0, 4, 8, 12) on different banks, so a warp's stores
  // are conflict-free (unswizzled: 4-way conflicts).  The swizzle keeps aligned
  // 4-column groups whole, so the GEMM's float4 reads stay single accesses.
  auto store_a_rows = [&](int buf) {
    const int sw = (tid & 3) << 3;  // swz(ak + j) for j < 4
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int col = (ar + 32 * i) ^ sw;
      As[buf][ak + 0][col] = areg[i].x;
      As[buf][ak + 1][col] = areg[i].y;
      As[buf][ak + 2][col] = areg[i].z;
      As[buf][ak + 3][col] = areg[i].w;
    }
  };
  // k-major A [K][M] and B [K][N] tiles by cp.async (zero-filled outside)
  auto copy_kmajor = [&](int64_t k0, int buf) {
    if (A_KMAJOR) {
#pragma unroll
      for (int i = 0; i < (kGemmBK * kGemmBM / 4) / kGemmThreads; ++i) {
        const int q = tid + i * kGemmThreads;
        const int kk = q / (kGemmBM / 4), mm = (q % (kGemmBM / 4)) * 4;
        const int64_t k = k0 + kk, m = m0 + mm;
        const bool ok = k < kend && m + 3 < G.M;
        sg_cp16(&As[buf][kk][mm], ok ? G.A + k * G.lda + m : G.A, ok);
      }
    }
#pragma unroll
    for (int i = 0; i < (kGemmBK * kGemmBN / 4) / kGemmThreads; ++i) {
      const int q = tid + i * kGemmThreads;
      const int kk = q / (kGemmBN / 4), nn = (q % (kGemmBN / 4)) * 4;
      const int64_t k = k0 + kk, n = n0 + nn;
      const bool ok = k < kend && n + 3 < G.N;
      sg_cp16(&Bs[buf][kk][nn], ok ? G.B + k * G.ldb + n : G.B, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  float2 acc[8][4];  // paired along the columns
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.f, 0.f);

  if (nsteps > 0) {
    if (!A_KMAJOR) {
      load_a_rows(kbeg);
      store_a_rows(0);
    }
    copy_kmajor(kbeg, 0);
  }
  for (int64_t step = 0; step < nsteps; ++step) {
    const int buf = static_cast<int>(step & 1);
    const bool more = step + 1 < nsteps;
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // tile `step` visible; buffer buf ^ 1 free
    if (more) {
      copy_kmajor(kbeg + (step + 1) * kGemmBK, buf ^ 1);
      if (!A_KMAJOR) load_a_rows(kbeg + (step + 1) * kGemmBK);
    }
#pragma unroll
    for (int kk = 0; kk < kGemmBK; ++kk) {
      const int sw = A_KMAJOR ? 0 : ((kk >> 2) & 3) << 3;  // swz(kk) of the [M][K] variant
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][(tm * 4) ^ sw]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][(64 + tm * 4) ^ sw]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tn * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][32 + tn * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float2 bv[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w),
                            make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma2(av[i], bv[j], acc[i][j]);
    }
    if (more && !A_KMAJOR) store_a_rows(buf ^ 1);
  }
  float* C = G.C + static_cast<int64_t>(blockIdx.z) * G.c_chunk_stride;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + (i < 4 ? tm * 4 + i : 64 + tm * 4 + i - 4);
    if (m >= G.M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t n = n0 + (j < 4 ? tn * 4 + j : 32 + tn * 4 + j - 4);
      if (n < G.N) C[m * G.ldc + n] = pair_at(acc[i], j);
    }
  }
}

}  // namespace ictc
