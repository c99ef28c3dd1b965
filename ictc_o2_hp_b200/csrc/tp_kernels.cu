// Fused FP32 TensorProduct forward and first-order VJP for sm_100a.
//
// Mapping.  Every output channel c of every path reads channel c of each input
// (cyclic routing, native_o2.py:128-129), so one row and one channel form a
// closed problem over a small "slot" vector (o2_paths.cuh).  A warp owns one row
// and a group of channels; consecutive lanes take consecutive channels, so each
// key segment is read and written with coalesced 4- or 8-byte accesses.  In full
// parity the two reflection copies ("worlds") of a channel sit in the two half
// warps (lanes 0-15: copy 0, lanes 16-31: copy 1) and run the same frequency-
// output paths in lockstep; only the scalar-output paths (world 0) diverge.
//
// A warp keeps the same channel group for its whole life, so its path weights
// stay in registers in the forward pass and its weight-gradient accumulators
// stay in registers in the backward pass.  The weight gradient is reduced
// deterministically: every warp "slot" writes one partial row, then a second
// kernel sums the slots in a fixed order (reference: two-stage FP32 reduction,
// triton_o2.py:744-780, 948-959).
//
// Two kernel families share this per-row arithmetic:
//   * staged: persistent CTAs (one per SM, two for small orders) that stream blocks of
//     whole rows into shared memory with bulk asynchronous copies (TMA) through an
//     mbarrier ring, so HBM latency hides behind the arithmetic of earlier rows; the
//     row-paired backward carries two rows per warp as f32x2 halves;
//   * direct: plain coalesced global loads, for operands that are not 16-byte
//     aligned or rows wider than one CTA.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <mutex>

#include "common.cuh"
#include "o2_paths.cuh"
#include "tma.cuh"
#include "tmap.cuh"

namespace ictc {

namespace {

constexpr int kDirectThreads = 128;  // 4 warps per CTA (direct kernels)
constexpr int kStagedWarps = 8;      // max warps of a staged CTA
constexpr size_t kStagedSmemBudget = 220 * 1024;
constexpr int kBarrierBytes = 128;   // mbarrier area at the start of dynamic smem
constexpr int kMaxStages = 4;

// ------------------------------------------------------------ memory helpers

__device__ __forceinline__ float2 ldg2(const float* p, bool vec2) {
  if (vec2) return __ldg(reinterpret_cast<const float2*>(p));
  return make_float2(__ldg(p), __ldg(p + 1));
}

// Read-only load the compiler may not hoist out of the row loop: keeping the
// loop-invariant path weights in registers would exceed the register budget of
// the backward kernel, whose registers hold the weight-gradient accumulators.
__device__ __forceinline__ float ld_stream(const float* p) {
  float v;
  asm volatile("ld.global.nc.L1::evict_last.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void st2(float* p, float a, float b, bool vec2) {
  if (vec2) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
  } else {
    p[0] = a;
    p[1] = b;
  }
}

// Source of a row's values: global memory (read-only path) or a shared-memory
// copy of the row.
struct GlobalRow {
  const float* p;
  bool vec2;
  __device__ __forceinline__ float ld(int i) const { return __ldg(p + i); }
  __device__ __forceinline__ float2 ld2(int i) const { return ldg2(p + i, vec2); }
};

// Explicit ld.shared (a generic load of shared memory costs more and waits on the
// long scoreboard); volatile keeps them after the mbarrier wait that publishes
// the stage.
struct SharedRow {
  uint32_t base;  // shared-window byte address of the row
  __device__ __forceinline__ explicit SharedRow(const float* p)
      : base(static_cast<uint32_t>(__cvta_generic_to_shared(p))) {}
  __device__ __forceinline__ float ld(int i) const {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(base + 4u * i));
    return v;
  }
  __device__ __forceinline__ float2 ld2(int i) const {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(base + 4u * i));
    return v;
  }
};

// Per-thread float4 weight chunks (see prescale_kernel) in shared or global memory.
struct SharedChunks {
  uint32_t base;  // byte address of chunk 0 of this thread
  int stride;     // bytes between chunks of one thread
  __device__ __forceinline__ float4 ld(int k) const {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(base + static_cast<uint32_t>(k * stride)));
    return v;
  }
};

struct GlobalChunks {
  const float4* p;  // chunk 0 of this thread
  int T;            // float4 stride between chunks
  __device__ __forceinline__ float4 ld(int k) const { return __ldg(p + k * T); }
};

// Slot vector of channel c in world q, in the canonical basis: the odd copy
// (r0, r1) is read as (-r1, r0) (reference fast_o2.py:61-66).
template <int M, bool FULL, bool CM, class Row>
__device__ __forceinline__ void load_slots(const Row& row, const TpLayout& L, int c, int q,
                                           float (&v)[2 * M + 2]) {
  v[0] = row.ld(c);
  v[1] = FULL ? row.ld(L.C + c) : 0.0f;
  auto put = [&](int m, float2 r) {
    v[2 * m] = q ? -r.y : r.x;
    v[2 * m + 1] = q ? r.x : r.y;
  };
  if constexpr (CM) {  // component-major: the two components C apart (triton_o2.py:116-118)
#pragma unroll
    for (int m = 1; m <= M; ++m) {
      const int o = L.fbase + (m - 1) * L.fstride + 2 * q * L.C + c;
      put(m, make_float2(row.ld(o), row.ld(o + L.C)));
    }
  } else {
#pragma unroll
    for (int m = 1; m <= M; ++m) put(m, row.ld2(L.fbase + (m - 1) * L.fstride + 2 * (q * L.C + c)));
  }
}

// Writes the frequency slots of world q; the odd copy (v0, v1) is stored as
// (v1, -v0) (reference fast_o2.py:68-73).  Scalars are written by world 0.
template <int M, bool FULL, bool CM>
__device__ __forceinline__ void store_slots(float* __restrict__ row, const TpLayout& L, int c,
                                            int q, bool vec2, const float (&v)[2 * M + 2]) {
  if (q == 0) {
    row[c] = v[0];
    if (FULL) row[L.C + c] = v[1];
  }
  if constexpr (CM) {
#pragma unroll
    for (int m = 1; m <= M; ++m) {
      float* p = row + L.fbase + (m - 1) * L.fstride + 2 * q * L.C + c;
      p[0] = q ? v[2 * m + 1] : v[2 * m];
      p[L.C] = q ? -v[2 * m] : v[2 * m + 1];
    }
  } else {
#pragma unroll
    for (int m = 1; m <= M; ++m)
      st2(row + L.fbase + (m - 1) * L.fstride + 2 * (q * L.C + c), q ? v[2 * m + 1] : v[2 * m],
          q ? -v[2 * m] : v[2 * m + 1], vec2);
  }
}

// ------------------------------------------------------------ path arithmetic

// Index of the weight used by path I for channel c in world q.
template <int M, bool FULL, int I>
__device__ __forceinline__ int weight_index(int C, int c, int q) {
  constexpr ChanPath cp = Paths<M, FULL>::table.p[I];
  return cp.unit * C + (cp.copied ? q * C : 0) + c;
}

constexpr int slot_dim(int slot) { return slot >= 2 ? 2 : 1; }

// True when term T of path I is the first term that writes accumulator `which`
// of kind `role` (0: output component k, 1: first-input component i, 2: second-
// input component j), so it is a plain product rather than an FMA.
template <int M, bool FULL, int I, int T, int role>
constexpr bool first_term() {
  constexpr ChanPath cp = Paths<M, FULL>::table.p[I];
  for (int u = 0; u < T; ++u) {
    const int a = role == 0 ? cp.t[u].k : (role == 1 ? cp.t[u].i : cp.t[u].j);
    const int b = role == 0 ? cp.t[T].k : (role == 1 ? cp.t[T].i : cp.t[T].j);
    if (a == b) return false;
  }
  return true;
}

// acc (+)= sign * x * y, or acc = sign * x * y for the first term.
template <bool FIRST, int SIGN>
__device__ __forceinline__ void mac(float& acc, float x, float y) {
  if constexpr (FIRST) {
    acc = SIGN > 0 ? x * y : -(x * y);
  } else {
    acc = SIGN > 0 ? fmaf(x, y, acc) : fmaf(-x, y, acc);
  }
}

// Forward contribution of path I: o[out + k] += w * sum_terms sign * a_i * b_j.
template <int M, bool FULL, int I>
__device__ __forceinline__ void path_forward(const float* a, const float* b, float* o, float w) {
  using P = Paths<M, FULL>;
  constexpr ChanPath cp = P::table.p[I];
  float s[2];
  static_for<cp.nt>([&](auto T) {
    constexpr Term t = P::table.p[I].t[T];
    mac<first_term<M, FULL, I, T, 0>(), t.s>(s[t.k], a[P::table.p[I].in1 + t.i],
                                              b[P::table.p[I].in2 + t.j]);
  });
  o[cp.out] = fmaf(w, s[0], o[cp.out]);
  if constexpr (slot_dim(cp.out) == 2) o[cp.out + 1] = fmaf(w, s[1], o[cp.out + 1]);
}

// First-order adjoint of path I for one row: dx, dy and the weight-gradient
// accumulator.  Three algebraically equal factorizations; the cheapest for the
// path's shape is chosen at compile time:
//   form 0:   s_k = sum a b,  acc += g.s,  dx_i += (w g_k) b_j,  dy_j += (w g_k) a_i
//   form 1/2: t_i = sum b_j g_k,  u_j = sum a_i g_k,  dx += w t,  dy += w u,
//             acc += a.t (form 1) or b.u (form 2)
template <int M, bool FULL, int I>
__device__ __forceinline__ void path_vjp(const float* a, const float* b, const float* g,
                                         float* dx, float* dy, float& acc, float w) {
  using P = Paths<M, FULL>;
  constexpr ChanPath cp = P::table.p[I];
  constexpr int d1 = slot_dim(cp.in1), d2 = slot_dim(cp.in2), d3 = slot_dim(cp.out);
  constexpr int cost0 = 2 * d3 + 3 * cp.nt;
  constexpr int cost1 = 2 * cp.nt + 2 * d1 + d2;
  constexpr int cost2 = 2 * cp.nt + d1 + 2 * d2;
  if constexpr (cost0 <= cost1 && cost0 <= cost2) {
    float s[2];
    static_for<cp.nt>([&](auto T) {
      constexpr Term t = P::table.p[I].t[T];
      mac<first_term<M, FULL, I, T, 0>(), t.s>(s[t.k], a[P::table.p[I].in1 + t.i],
                                                b[P::table.p[I].in2 + t.j]);
    });
    float wg[2];
    acc = fmaf(g[cp.out], s[0], acc);
    wg[0] = w * g[cp.out];
    if constexpr (d3 == 2) {
      acc = fmaf(g[cp.out + 1], s[1], acc);
      wg[1] = w * g[cp.out + 1];
    }
    static_for<cp.nt>([&](auto T) {
      constexpr Term t = P::table.p[I].t[T];
      constexpr int i1 = P::table.p[I].in1 + t.i;
      constexpr int i2 = P::table.p[I].in2 + t.j;
      mac<false, t.s>(dx[i1], wg[t.k], b[i2]);
      mac<false, t.s>(dy[i2], wg[t.k], a[i1]);
    });
  } else {
    float tv[2], uv[2];
    static_for<cp.nt>([&](auto T) {
      constexpr Term t = P::table.p[I].t[T];
      constexpr int i1 = P::table.p[I].in1 + t.i;
      constexpr int i2 = P::table.p[I].in2 + t.j;
      constexpr int i3 = P::table.p[I].out + t.k;
      mac<first_term<M, FULL, I, T, 1>(), t.s>(tv[t.i], b[i2], g[i3]);
      mac<first_term<M, FULL, I, T, 2>(), t.s>(uv[t.j], a[i1], g[i3]);
    });
    static_for<d1>([&](auto i) { dx[cp.in1 + i] = fmaf(w, tv[i], dx[cp.in1 + i]); });
    static_for<d2>([&](auto j) { dy[cp.in2 + j] = fmaf(w, uv[j], dy[cp.in2 + j]); });
    if constexpr (cost1 <= cost2) {
      static_for<d1>([&](auto i) { acc = fmaf(a[cp.in1 + i], tv[i], acc); });
    } else {
      static_for<d2>([&](auto j) { acc = fmaf(b[cp.in2 + j], uv[j], acc); });
    }
  }
}

// Loads the register-resident path weights of (channel c, world q), magnitude
// folded in.  Unused entries (scalar-output paths in world 1) are zero.
template <int M, bool FULL>
__device__ __forceinline__ void load_weights(const float* __restrict__ w, const TpLayout& L,
                                             const Mags& mags, int c, int q, bool active,
                                             float (&wr)[Paths<M, FULL>::n]) {
  using P = Paths<M, FULL>;
  static_for<P::n>([&](auto I) {
    constexpr ChanPath cp = P::table.p[I];
    const bool used = active && (!FULL || cp.copied || q == 0);
    wr[I] = used ? __ldg(w + weight_index<M, FULL, I>(L.C, c, q)) * mags.m[cp.cls] : 0.0f;
  });
}

// Forward of one (row, channel, world): o = sum over paths, in Paths::vjp order
// (the scalar-output paths of world 0 form one divergent region).
template <int M, bool FULL>
__device__ __forceinline__ void row_forward(const float (&a)[2 * M + 2],
                                            const float (&b)[2 * M + 2],
                                            const float (&wr)[Paths<M, FULL>::n], int q,
                                            float (&o)[2 * M + 2]) {
  using P = Paths<M, FULL>;
#pragma unroll
  for (int s = 0; s < 2 * M + 2; ++s) o[s] = 0.0f;
  auto step = [&](auto K) {
    constexpr int I = P::vjp.idx[K];
    path_forward<M, FULL, I>(a, b, o, wr[I]);
  };
  static_for<P::nfreq>(step);
  if (!FULL || q == 0) {
    static_for<P::n - P::nfreq>([&](auto J) { step(std::integral_constant<int, P::nfreq + J>{}); });
  }
}

// VJP of one (row, channel, world).  Paths run in Paths::vjp order (frequency-
// output paths, then the world-0 scalar-output paths); the magnitude-scaled
// weights of this thread sit in that order as float4 chunks (prescale_kernel).
template <int M, bool FULL, class Chunks>
__device__ __forceinline__ void row_vjp(const float (&a)[2 * M + 2], const float (&b)[2 * M + 2],
                                        const float (&g)[2 * M + 2], const Chunks& wsrc, int q,
                                        float (&dx)[2 * M + 2], float (&dy)[2 * M + 2],
                                        float (&acc)[Paths<M, FULL>::n]) {
  using P = Paths<M, FULL>;
#pragma unroll
  for (int s = 0; s < 2 * M + 2; ++s) {
    dx[s] = 0.0f;
    dy[s] = 0.0f;
  }
  float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
  auto step = [&](auto K) {
    constexpr int I = P::vjp.idx[K];
    if constexpr (K % 4 == 0) w4 = wsrc.ld(K / 4);
    const float wv = K % 4 == 0 ? w4.x : (K % 4 == 1 ? w4.y : (K % 4 == 2 ? w4.z : w4.w));
    path_vjp<M, FULL, I>(a, b, g, dx, dy, acc[K], wv);
  };
  static_for<P::nfreq>(step);
  if (!FULL || q == 0) {  // scalar-output paths: world 0 only
    static_for<P::n - P::nfreq>([&](auto J) { step(std::integral_constant<int, P::nfreq + J>{}); });
  }
  if (FULL) {
    // World 1 reaches the scalars through scalar x frequency paths.
    dx[0] += __shfl_xor_sync(0xffffffffu, dx[0], 16);
    dx[1] += __shfl_xor_sync(0xffffffffu, dx[1], 16);
    dy[0] += __shfl_xor_sync(0xffffffffu, dy[0], 16);
    dy[1] += __shfl_xor_sync(0xffffffffu, dy[1], 16);
  }
}

// Writes the weight-gradient accumulators of one thread (in Paths::vjp order)
// to its partial row.
template <int M, bool FULL>
__device__ __forceinline__ void store_partial(float* __restrict__ dst, const TpLayout& L,
                                              const Mags& mags, int c, int q,
                                              const float (&acc)[Paths<M, FULL>::n]) {
  using P = Paths<M, FULL>;
  static_for<P::n>([&](auto K) {
    constexpr int I = P::vjp.idx[K];
    constexpr ChanPath cp = P::table.p[I];
    if (FULL && !cp.copied && q != 0) return;
    dst[weight_index<M, FULL, I>(L.C, c, q)] = acc[K] * mags.m[cp.cls];
  });
}

// ------------------------------------------------------------ row-paired adjoint
//
// Two rows of the same (channel, world) run the same paths with the same weights and
// signs, so the backward can carry them as the two halves of f32x2 values: every
// product and dx / dy update of both rows is one paired FMA (each half rounded
// exactly as the scalar form), and only the weight-gradient accumulator, shared by
// the rows, takes two scalar FMAs.

template <bool FIRST, int SIGN>
__device__ __forceinline__ void mac2(float2& acc, float2 x, float2 y) {
  if constexpr (FIRST) {
    acc = SIGN > 0 ? __fmul2_rn(x, y) : __fmul2_rn(make_float2(-x.x, -x.y), y);
  } else {
    acc = SIGN > 0 ? __ffma2_rn(x, y, acc) : __ffma2_rn(make_float2(-x.x, -x.y), y, acc);
  }
}

__device__ __forceinline__ float2 fma2w(float w, float2 x, float2 acc) {
  return __ffma2_rn(make_float2(w, w), x, acc);
}

// path_vjp for a row pair (same factorizations, chosen the same way).
template <int M, bool FULL, int I>
__device__ __forceinline__ void path_vjp2(const float2* a, const float2* b, const float2* g,
                                          float2* dx, float2* dy, float& acc, float w) {
  using P = Paths<M, FULL>;
  constexpr ChanPath cp = P::table.p[I];
  constexpr int d1 = slot_dim(cp.in1), d2 = slot_dim(cp.in2), d3 = slot_dim(cp.out);
  constexpr int cost0 = 2 * d3 + 3 * cp.nt;
  constexpr int cost1 = 2 * cp.nt + 2 * d1 + d2;
  constexpr int cost2 = 2 * cp.nt + d1 + 2 * d2;
  if constexpr (cost0 <= cost1 && cost0 <= cost2) {
    float2 s[2];
    static_for<cp.nt>([&](auto T) {
      constexpr Term t = P::table.p[I].t[T];
      mac2<first_term<M, FULL, I, T, 0>(), t.s>(s[t.k], a[P::table.p[I].in1 + t.i],
                                                 b[P::table.p[I].in2 + t.j]);
    });
    float2 wg[2];
    acc = fmaf(g[cp.out].x, s[0].x, acc);
    acc = fmaf(g[cp.out].y, s[0].y, acc);
    wg[0] = __fmul2_rn(make_float2(w, w), g[cp.out]);
    if constexpr (d3 == 2) {
      acc = fmaf(g[cp.out + 1].x, s[1].x, acc);
      acc = fmaf(g[cp.out + 1].y, s[1].y, acc);
      wg[1] = __fmul2_rn(make_float2(w, w), g[cp.out + 1]);
    }
    static_for<cp.nt>([&](auto T) {
      constexpr Term t = P::table.p[I].t[T];
      constexpr int i1 = P::table.p[I].in1 + t.i;
      constexpr int i2 = P::table.p[I].in2 + t.j;
      mac2<false, t.s>(dx[i1], wg[t.k], b[i2]);
      mac2<false, t.s>(dy[i2], wg[t.k], a[i1]);
    });
  } else {
    float2 tv[2], uv[2];
    static_for<cp.nt>([&](auto T) {
      constexpr Term t = P::table.p[I].t[T];
      constexpr int i1 = P::table.p[I].in1 + t.i;
      constexpr int i2 = P::table.p[I].in2 + t.j;
      constexpr int i3 = P::table.p[I].out + t.k;
      mac2<first_term<M, FULL, I, T, 1>(), t.s>(tv[t.i], b[i2], g[i3]);
      mac2<first_term<M, FULL, I, T, 2>(), t.s>(uv[t.j], a[i1], g[i3]);
    });
    static_for<d1>([&](auto i) { dx[cp.in1 + i] = fma2w(w, tv[i], dx[cp.in1 + i]); });
    static_for<d2>([&](auto j) { dy[cp.in2 + j] = fma2w(w, uv[j], dy[cp.in2 + j]); });
    if constexpr (cost1 <= cost2) {
      static_for<d1>([&](auto i) {
        acc = fmaf(a[cp.in1 + i].x, tv[i].x, acc);
        acc = fmaf(a[cp.in1 + i].y, tv[i].y, acc);
      });
    } else {
      static_for<d2>([&](auto j) {
        acc = fmaf(b[cp.in2 + j].x, uv[j].x, acc);
        acc = fmaf(b[cp.in2 + j].y, uv[j].y, acc);
      });
    }
  }
}

// row_vjp for a row pair.
template <int M, bool FULL, class Chunks>
__device__ __forceinline__ void row_vjp2(const float2 (&a)[2 * M + 2],
                                         const float2 (&b)[2 * M + 2],
                                         const float2 (&g)[2 * M + 2], const Chunks& wsrc, int q,
                                         float2 (&dx)[2 * M + 2], float2 (&dy)[2 * M + 2],
                                         float (&acc)[Paths<M, FULL>::n]) {
  using P = Paths<M, FULL>;
#pragma unroll
  for (int s = 0; s < 2 * M + 2; ++s) {
    dx[s] = make_float2(0.f, 0.f);
    dy[s] = make_float2(0.f, 0.f);
  }
  float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
  auto step = [&](auto K) {
    constexpr int I = P::vjp.idx[K];
    if constexpr (K % 4 == 0) w4 = wsrc.ld(K / 4);
    const float wv = K % 4 == 0 ? w4.x : (K % 4 == 1 ? w4.y : (K % 4 == 2 ? w4.z : w4.w));
    path_vjp2<M, FULL, I>(a, b, g, dx, dy, acc[K], wv);
  };
  static_for<P::nfreq>(step);
  if (!FULL || q == 0) {
    static_for<P::n - P::nfreq>([&](auto J) { step(std::integral_constant<int, P::nfreq + J>{}); });
  }
  if (FULL) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      dx[s].x += __shfl_xor_sync(0xffffffffu, dx[s].x, 16);
      dx[s].y += __shfl_xor_sync(0xffffffffu, dx[s].y, 16);
      dy[s].x += __shfl_xor_sync(0xffffffffu, dy[s].x, 16);
      dy[s].y += __shfl_xor_sync(0xffffffffu, dy[s].y, 16);
    }
  }
}

// Lane -> (channel, world) of a warp that owns channel group `group`.
template <bool FULL>
struct LaneMap {
  int q, c;
  bool active;
  __device__ __forceinline__ LaneMap(int group, int lane, int C) {
    constexpr int CPW = FULL ? 16 : 32;
    q = FULL ? (lane >> 4) : 0;
    const int raw = group * CPW + (FULL ? (lane & 15) : lane);
    active = raw < C;
    c = active ? raw : 0;  // inactive lanes compute on channel 0 and store nothing
  }
};

// ------------------------------------------------------------ direct kernels

template <int M, bool FULL, bool CM = false>
__global__ void __launch_bounds__(kDirectThreads)
    tp_forward_direct(const float* __restrict__ x, const float* __restrict__ y,
                      const float* __restrict__ w, float* __restrict__ out, int64_t rows,
                      TpLayout L, Mags mags, int groups, int64_t nwarps, int64_t slots,
                      bool vec2) {
  constexpr int S = 2 * M + 2;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (gw >= nwarps) return;
  const LaneMap<FULL> lm(static_cast<int>(gw % groups), lane, L.C);
  float wr[Paths<M, FULL>::n];
  load_weights<M, FULL>(w, L, mags, lm.c, lm.q, lm.active, wr);
  for (int64_t row = gw / groups; row < rows; row += slots) {
    float a[S], b[S], o[S];
    load_slots<M, FULL, CM>(GlobalRow{x + row * L.width, vec2}, L, lm.c, lm.q, a);
    load_slots<M, FULL, CM>(GlobalRow{y + row * L.width, vec2}, L, lm.c, lm.q, b);
    row_forward<M, FULL>(a, b, wr, lm.q, o);
    if (lm.active) store_slots<M, FULL, CM>(out + row * L.width, L, lm.c, lm.q, vec2, o);
  }
}

template <int M, bool FULL, bool CM = false>
__global__ void __launch_bounds__(kDirectThreads)
    tp_backward_direct(const float* __restrict__ x, const float* __restrict__ y,
                       const float4* __restrict__ ws, const float* __restrict__ go,
                       float* __restrict__ gx, float* __restrict__ gy,
                       float* __restrict__ partial, int64_t numel, int64_t rows, TpLayout L,
                       Mags mags, int groups, int64_t nwarps, int64_t slots, bool vec2) {
  using P = Paths<M, FULL>;
  constexpr int S = 2 * M + 2;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (gw >= nwarps) return;  // whole warps only: nwarps counts warps
  const LaneMap<FULL> lm(static_cast<int>(gw % groups), lane, L.C);
  const int64_t slot = gw / groups;
  float acc[P::n];
#pragma unroll
  for (int i = 0; i < P::n; ++i) acc[i] = 0.0f;
  for (int64_t row = slot; row < rows; row += slots) {
    float a[S], b[S], g[S], dx[S], dy[S];
    load_slots<M, FULL, CM>(GlobalRow{x + row * L.width, vec2}, L, lm.c, lm.q, a);
    load_slots<M, FULL, CM>(GlobalRow{y + row * L.width, vec2}, L, lm.c, lm.q, b);
    // The output twist (v0, v1) -> (v1, -v0) has the adjoint g -> (-g1, g0),
    // which is the same map as the input read.
    load_slots<M, FULL, CM>(GlobalRow{go + row * L.width, vec2}, L, lm.c, lm.q, g);
    const GlobalChunks chunks{ws + static_cast<int>(gw % groups) * 32 + lane, groups * 32};
    row_vjp<M, FULL>(a, b, g, chunks, lm.q, dx, dy, acc);
    if (lm.active) {
      store_slots<M, FULL, CM>(gx + row * L.width, L, lm.c, lm.q, vec2, dx);
      store_slots<M, FULL, CM>(gy + row * L.width, L, lm.c, lm.q, vec2, dy);
    }
  }
  if (lm.active) store_partial<M, FULL>(partial + slot * numel, L, mags, lm.c, lm.q, acc);
}

// ------------------------------------------------------------ staged kernels
//
// A CTA of R * groups warps; warp (r, g) handles row r of each stage and channel
// group g.  A stage holds NT tensors of R consecutive rows (contiguous in HBM, one
// bulk copy each).  Thread 0 issues copies: `stages` blocks up front, then it
// refills the stage consumed one iteration earlier once every warp has released
// it.  Blocks of rows are dealt round-robin over the persistent grid.

struct StageRing {
  uint64_t* full;
  uint64_t* empty;
  float* buf;
};

// Barriers live in the first kBarrierBytes of `smem`; stage buffers start at
// `base + kBarrierBytes` (base = smem, or past data placed in front of them).
__device__ __forceinline__ StageRing stage_ring(unsigned char* smem, unsigned char* base,
                                                int stages) {
  StageRing ring;
  ring.full = reinterpret_cast<uint64_t*>(smem);
  ring.empty = ring.full + stages;
  ring.buf = reinterpret_cast<float*>(base + kBarrierBytes);
  return ring;
}

template <int NT>
__device__ __forceinline__ void issue_stage(const StageRing& ring, int s, int64_t block, int R,
                                            int64_t rows, int64_t W, const float* const* src) {
  const int64_t row0 = block * R;
  const int64_t nr = rows - row0 < R ? rows - row0 : R;
  const uint32_t bytes = static_cast<uint32_t>(nr * W * 4);
  float* dst = ring.buf + static_cast<int64_t>(s) * NT * R * W;
  mbar_arrive_expect_tx(&ring.full[s], NT * bytes);
#pragma unroll
  for (int t = 0; t < NT; ++t) bulk_g2s(dst + t * R * W, src[t] + row0 * W, bytes, &ring.full[s]);
}

// Pipeline driver: calls body(stage_base, row) for every row of this CTA's
// blocks (row < rows), with the whole stage resident in shared memory.  Each
// warp counts itself out of a stage when done with it (acquire-release atomic
// on a per-stage counter); the warp that completes the count refills the stage
// at once, so no warp ever blocks waiting for the others to release a stage.
// COUNT: the stage index and its fill round are carried from block to block (the
// backward: 0.946 -> 0.908 ms at TP(128, 6, full), 65,536 rows) or recomputed from the
// block count by division (the forwards: 0.462 ms against 0.470 ms with counters).
template <int NT, bool COUNT, int RPW = 1, class Body>
__device__ __forceinline__ void staged_loop(unsigned char* smem, unsigned char* base, int stages,
                                            int R, int64_t rows, int64_t W,
                                            const float* const* src, Body&& body) {
  const StageRing ring = stage_ring(smem, base, stages);
  // the counters live where the stages' "empty" barriers would be
  unsigned* done = reinterpret_cast<unsigned*>(ring.empty);
  const int nwarps = blockDim.x >> 5;
  const int r = (threadIdx.x >> 5) / (nwarps / R);
  const int RB = R * RPW;  // rows per block: RPW per warp row slot
  const int64_t nblocks = (rows + RB - 1) / RB;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&ring.full[s], 1);
      done[s] = 0;
    }
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      const int64_t block = blockIdx.x + static_cast<int64_t>(s) * gridDim.x;
      if (block < nblocks) issue_stage<NT>(ring, s, block, RB, rows, W, src);
    }
  }
  int s = 0;
  uint32_t round = 0;
  int64_t it = 0;
  bool ok = true;
  for (int64_t block = blockIdx.x; block < nblocks && ok; block += gridDim.x, ++it) {
    if constexpr (!COUNT) {
      s = static_cast<int>(it % stages);
      round = static_cast<uint32_t>(it / stages);
    }
    ok = mbar_wait(&ring.full[s], round & 1, 1);
    if (!ok) break;
    const int64_t row = block * RB + r * RPW;
    if (row < rows) body(ring.buf + static_cast<int64_t>(s) * NT * RB * W + r * RPW * W, row);
    __syncwarp();
    if ((threadIdx.x & 31) == 0) {
      unsigned prev;
      asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                   : "=r"(prev)
                   : "r"(smem_addr(&done[s]))
                   : "memory");
      if (prev + 1 == static_cast<unsigned>(nwarps) * (round + 1)) {
        // every warp is done reading stage s: order those reads before the
        // asynchronous copy that overwrites it, then refill
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const int64_t next = block + static_cast<int64_t>(stages) * gridDim.x;
        if (next < nblocks) issue_stage<NT>(ring, s, next, RB, rows, W, src);
      }
    }
    if constexpr (COUNT) {
      if (++s == stages) {
        s = 0;
        ++round;
      }
    }
  }
  if (!ok && threadIdx.x == 0) {
    // a wait ran out: let copies already issued land before the CTA exits
    for (int st = 0; st < stages; ++st) mbar_wait(&ring.full[st], 0, 3, kDrainLimitNs);
  }
}

template <int M, bool FULL, bool CM = false>
__global__ void __launch_bounds__(kStagedWarps * 32, 1)
    tp_forward_staged(const float* __restrict__ x, const float* __restrict__ y,
                      const float* __restrict__ w, float* __restrict__ out, int64_t rows,
                      TpLayout L, Mags mags, int groups, int R, int stages) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int S = 2 * M + 2;
  const int warp = threadIdx.x >> 5;
  const LaneMap<FULL> lm(warp % groups, threadIdx.x & 31, L.C);
  float wr[Paths<M, FULL>::n];
  load_weights<M, FULL>(w, L, mags, lm.c, lm.q, lm.active, wr);
  const float* src[2] = {x, y};
  const int64_t W = L.width;
  staged_loop<2, false>(smem, smem, stages, R, rows, W, src, [&](const float* stage, int64_t row) {
    float a[S], b[S], o[S];
    load_slots<M, FULL, CM>(SharedRow(stage), L, lm.c, lm.q, a);
    load_slots<M, FULL, CM>(SharedRow(stage + R * W), L, lm.c, lm.q, b);
    row_forward<M, FULL>(a, b, wr, lm.q, o);
    if (lm.active) store_slots<M, FULL, CM>(out + row * W, L, lm.c, lm.q, true, o);
  });
}

// The magnitude-scaled path weights of thread t (channel lm.c, world lm.q) as float4
// chunks in Paths::vjp order, chunk k at wsm[k * T + t] (T threads per row); unused
// entries (scalar-output paths of world 1, inactive lanes, the last chunk's tail) are 0.
template <int M, bool FULL>
__device__ __forceinline__ void build_weight_chunks(const float* __restrict__ w,
                                                    const TpLayout& L, const Mags& mags,
                                                    const LaneMap<FULL>& lm, int T, int t,
                                                    float4* wsm) {
  using P = Paths<M, FULL>;
  static_for<P::chunks>([&](auto k) {
    float v[4];
    static_for<4>([&](auto e) {
      constexpr int pos = 4 * k + e;
      if constexpr (pos < P::n) {
        constexpr int I = P::vjp.idx[pos];
        constexpr ChanPath cp = P::table.p[I];
        const bool used = lm.active && (!FULL || cp.copied || lm.q == 0);
        v[e] = used ? __ldg(w + weight_index<M, FULL, I>(L.C, lm.c, lm.q)) * mags.m[cp.cls]
                    : 0.0f;
      } else {
        v[e] = 0.0f;
      }
    });
    wsm[k * T + t] = make_float4(v[0], v[1], v[2], v[3]);
  });
}

// Forward with the path weights in shared memory instead of registers: with
// register use capped at 128, CTAs of 16 warps (two rows per stage) fit on an SM,
// twice the warps of the register-weight variant.  The weights are laid out as
// per-thread float4 chunks (thread t, chunk k at [k * T + t], Paths::vjp order)
// by the warps of row slot 0 at kernel start.
constexpr int kWideWarps = 16;

template <int M, bool FULL>
constexpr size_t wide_forward_smem() {
  // worst case over channel counts: 256 threads per row, R * W <= 512 (2M + 1)
  return kBarrierBytes + static_cast<size_t>(Paths<M, FULL>::chunks) * 256 * 16 +
         2 * 2 * static_cast<size_t>(FULL ? 512 : 256) * (2 * M + 1) * 4;
}

template <int M, bool FULL>
constexpr bool wide_forward_fits() { return wide_forward_smem<M, FULL>() <= kStagedSmemBudget; }

template <int M, bool FULL, bool CM = false>
__global__ void __launch_bounds__(kWideWarps * 32, 1)
    tp_forward_wide(const float* __restrict__ x, const float* __restrict__ y,
                    const float* __restrict__ w, float* __restrict__ out, int64_t rows,
                    TpLayout L, Mags mags, int groups, int R, int stages) {
  extern __shared__ __align__(128) unsigned char smem[];
  using P = Paths<M, FULL>;
  constexpr int S = 2 * M + 2;
  const int warp = threadIdx.x >> 5;
  const int T = groups * 32;
  const int t = (warp % groups) * 32 + (threadIdx.x & 31);
  const LaneMap<FULL> lm(warp % groups, threadIdx.x & 31, L.C);
  float4* wsm = reinterpret_cast<float4*>(smem + kBarrierBytes);
  if (warp < groups) build_weight_chunks<M, FULL>(w, L, mags, lm, T, t, wsm);
  __syncthreads();
  const SharedChunks chunks{static_cast<uint32_t>(__cvta_generic_to_shared(wsm + t)),
                            T * static_cast<int>(sizeof(float4))};
  const size_t wbytes = static_cast<size_t>(P::chunks) * T * sizeof(float4);
  const float* src[2] = {x, y};
  const int64_t W = L.width;
  staged_loop<2, false>(smem, smem + wbytes, stages, R, rows, W, src,
                        [&](const float* stage, int64_t row) {
    float a[S], b[S], o[S];
    load_slots<M, FULL, CM>(SharedRow(stage), L, lm.c, lm.q, a);
    load_slots<M, FULL, CM>(SharedRow(stage + R * W), L, lm.c, lm.q, b);
#pragma unroll
    for (int i = 0; i < S; ++i) o[i] = 0.0f;
    float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
    auto step = [&](auto K) {
      constexpr int I = P::vjp.idx[K];
      if constexpr (K % 4 == 0) w4 = chunks.ld(K / 4);
      const float wv = K % 4 == 0 ? w4.x : (K % 4 == 1 ? w4.y : (K % 4 == 2 ? w4.z : w4.w));
      path_forward<M, FULL, I>(a, b, o, wv);
    };
    static_for<P::nfreq>(step);
    if (!FULL || lm.q == 0) {
      static_for<P::n - P::nfreq>(
          [&](auto J) { step(std::integral_constant<int, P::nfreq + J>{}); });
    }
    if (lm.active) store_slots<M, FULL, CM>(out + row * W, L, lm.c, lm.q, true, o);
  });
}

// path_forward for a row pair: the two rows are the halves of float2 values, so each
// product and output update is one paired FMA, each half rounded exactly as the
// scalar form (bit-identical per row).
template <int M, bool FULL, int I>
__device__ __forceinline__ void path_forward2(const float2* a, const float2* b, float2* o,
                                              float w) {
  using P = Paths<M, FULL>;
  constexpr ChanPath cp = P::table.p[I];
  float2 s[2];
  static_for<cp.nt>([&](auto T) {
    constexpr Term t = P::table.p[I].t[T];
    mac2<first_term<M, FULL, I, T, 0>(), t.s>(s[t.k], a[P::table.p[I].in1 + t.i],
                                               b[P::table.p[I].in2 + t.j]);
  });
  o[cp.out] = fma2w(w, s[0], o[cp.out]);
  if constexpr (slot_dim(cp.out) == 2) o[cp.out + 1] = fma2w(w, s[1], o[cp.out + 1]);
}

// tp_forward_wide on row pairs: each warp takes two rows per stage block (the halves of
// its float2 operands), half the FMA instructions per row, on CTAs of kWidePairWarps
// warps (no register cap below 255: the pair state is three float2 rows of slots).
// A missing second row (odd row count) computes on zeros and stores nothing.
constexpr int kWidePairWarps = 8;

template <int M, bool FULL, bool CM = false>
__global__ void __launch_bounds__(kWidePairWarps * 32, 1)
    tp_forward_wide_paired(const float* __restrict__ x, const float* __restrict__ y,
                           const float* __restrict__ w, float* __restrict__ out, int64_t rows,
                           TpLayout L, Mags mags, int groups, int R, int stages) {
  extern __shared__ __align__(128) unsigned char smem[];
  using P = Paths<M, FULL>;
  constexpr int S = 2 * M + 2;
  const int warp = threadIdx.x >> 5;
  const int T = groups * 32;
  const int t = (warp % groups) * 32 + (threadIdx.x & 31);
  const LaneMap<FULL> lm(warp % groups, threadIdx.x & 31, L.C);
  float4* wsm = reinterpret_cast<float4*>(smem + kBarrierBytes);
  if (warp < groups) build_weight_chunks<M, FULL>(w, L, mags, lm, T, t, wsm);
  __syncthreads();
  const SharedChunks chunks{static_cast<uint32_t>(__cvta_generic_to_shared(wsm + t)),
                            T * static_cast<int>(sizeof(float4))};
  const size_t wbytes = static_cast<size_t>(P::chunks) * T * sizeof(float4);
  const float* src[2] = {x, y};
  const int64_t W = L.width;
  const int RB = 2 * R;  // rows per stage block
  staged_loop<2, false, 2>(smem, smem + wbytes, stages, R, rows, W, src,
                           [&](const float* stage, int64_t row) {
    const bool two = row + 1 < rows;
    float2 a[S], b[S], o[S];
    auto load_pair = [&](const float* base, float2 (&v)[S]) {
      float u0[S], u1[S];
      load_slots<M, FULL, CM>(SharedRow(base), L, lm.c, lm.q, u0);
      load_slots<M, FULL, CM>(SharedRow(base + W), L, lm.c, lm.q, u1);
#pragma unroll
      for (int k = 0; k < S; ++k) v[k] = make_float2(u0[k], two ? u1[k] : 0.f);
    };
    load_pair(stage, a);
    load_pair(stage + RB * W, b);
#pragma unroll
    for (int i = 0; i < S; ++i) o[i] = make_float2(0.f, 0.f);
    float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
    auto step = [&](auto K) {
      constexpr int I = P::vjp.idx[K];
      if constexpr (K % 4 == 0) w4 = chunks.ld(K / 4);
      const float wv = K % 4 == 0 ? w4.x : (K % 4 == 1 ? w4.y : (K % 4 == 2 ? w4.z : w4.w));
      path_forward2<M, FULL, I>(a, b, o, wv);
    };
    static_for<P::nfreq>(step);
    if (!FULL || lm.q == 0) {
      static_for<P::n - P::nfreq>(
          [&](auto J) { step(std::integral_constant<int, P::nfreq + J>{}); });
    }
    if (lm.active) {
      float v0[S], v1[S];
#pragma unroll
      for (int k = 0; k < S; ++k) {
        v0[k] = o[k].x;
        v1[k] = o[k].y;
      }
      store_slots<M, FULL, CM>(out + row * W, L, lm.c, lm.q, true, v0);
      if (two) store_slots<M, FULL, CM>(out + (row + 1) * W, L, lm.c, lm.q, true, v1);
    }
  });
}

// Forward with the group's path weights in shared memory: a CTA of
// kGroupFwdWarps warps serves ONE channel group and its warps take rows round-
// robin, so the weights (float4 chunks in Paths::vjp order, built at start from
// the packed vector) cost 16 B x chunks per lane of shared memory instead of
// Paths::n registers.  The freed registers buy resident warps, which hide the
// latency of the coalesced global loads of x and y.
constexpr int kGroupFwdWarps = 4;

template <int M, bool FULL, bool CM = false>
__global__ void __launch_bounds__(kGroupFwdWarps * 32)
    tp_forward_grouped(const float* __restrict__ x, const float* __restrict__ y,
                       const float* __restrict__ w, float* __restrict__ out, int64_t rows,
                       TpLayout L, Mags mags, int groups, int64_t row_slots, bool vec2) {
  using P = Paths<M, FULL>;
  constexpr int S = 2 * M + 2;
  extern __shared__ __align__(16) float4 wsm[];  // [chunk][32 lanes]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int group = static_cast<int>(blockIdx.x % groups);
  const LaneMap<FULL> lm(group, lane, L.C);
  static_for<P::chunks>([&](auto k) {
    if (k % kGroupFwdWarps != warp) return;
    float v[4];
    static_for<4>([&](auto e) {
      constexpr int pos = 4 * k + e;
      if constexpr (pos < P::n) {
        constexpr int I = P::vjp.idx[pos];
        constexpr ChanPath cp = P::table.p[I];
        const bool used = lm.active && (!FULL || cp.copied || lm.q == 0);
        v[e] = used ? __ldg(w + weight_index<M, FULL, I>(L.C, lm.c, lm.q)) * mags.m[cp.cls]
                    : 0.0f;
      } else {
        v[e] = 0.0f;
      }
    });
    wsm[k * 32 + lane] = make_float4(v[0], v[1], v[2], v[3]);
  });
  __syncthreads();
  const SharedChunks chunks{static_cast<uint32_t>(__cvta_generic_to_shared(wsm + lane)),
                            32 * static_cast<int>(sizeof(float4))};
  const int64_t first = static_cast<int64_t>(blockIdx.x / groups) * kGroupFwdWarps + warp;
  for (int64_t row = first; row < rows; row += row_slots) {
    float a[S], b[S], o[S];
    load_slots<M, FULL, CM>(GlobalRow{x + row * L.width, vec2}, L, lm.c, lm.q, a);
    load_slots<M, FULL, CM>(GlobalRow{y + row * L.width, vec2}, L, lm.c, lm.q, b);
#pragma unroll
    for (int i = 0; i < S; ++i) o[i] = 0.0f;
    float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
    auto step = [&](auto K) {
      constexpr int I = P::vjp.idx[K];
      if constexpr (K % 4 == 0) w4 = chunks.ld(K / 4);
      const float wv = K % 4 == 0 ? w4.x : (K % 4 == 1 ? w4.y : (K % 4 == 2 ? w4.z : w4.w));
      path_forward<M, FULL, I>(a, b, o, wv);
    };
    static_for<P::nfreq>(step);
    if (!FULL || lm.q == 0) {
      static_for<P::n - P::nfreq>(
          [&](auto J) { step(std::integral_constant<int, P::nfreq + J>{}); });
    }
    if (lm.active) store_slots<M, FULL, CM>(out + row * L.width, L, lm.c, lm.q, vec2, o);
  }
}

template <int M, bool FULL, bool CM = false>
__global__ void __launch_bounds__(kStagedWarps * 32, 1)
    tp_backward_staged(const float* __restrict__ x, const float* __restrict__ y,
                       const float4* __restrict__ ws, const float* __restrict__ go,
                       float* __restrict__ gx, float* __restrict__ gy,
                       float* __restrict__ partial, int64_t numel, int64_t rows, TpLayout L,
                       Mags mags, int groups, int R, int stages, int weights_in_smem) {
  extern __shared__ __align__(128) unsigned char smem[];
  using P = Paths<M, FULL>;
  constexpr int S = 2 * M + 2;
  const int warp = threadIdx.x >> 5;
  const int r = warp / groups;
  const int T = groups * 32;
  const int t = (warp % groups) * 32 + (threadIdx.x & 31);
  const LaneMap<FULL> lm(warp % groups, threadIdx.x & 31, L.C);
  // Weights: copied once into shared memory when they fit next to the stages.
  const size_t wbytes = static_cast<size_t>(P::chunks) * T * sizeof(float4);
  float acc[P::n];
#pragma unroll
  for (int i = 0; i < P::n; ++i) acc[i] = 0.0f;
  const float* src[3] = {x, y, go};
  const int64_t W = L.width;
  auto body = [&](const auto& chunks) {
    return [&](const float* stage, int64_t row) {
      float a[S], b[S], g[S], dx[S], dy[S];
      load_slots<M, FULL, CM>(SharedRow(stage), L, lm.c, lm.q, a);
      load_slots<M, FULL, CM>(SharedRow(stage + R * W), L, lm.c, lm.q, b);
      load_slots<M, FULL, CM>(SharedRow(stage + 2 * R * W), L, lm.c, lm.q, g);
      row_vjp<M, FULL>(a, b, g, chunks, lm.q, dx, dy, acc);
      if (lm.active) {
        store_slots<M, FULL, CM>(gx + row * W, L, lm.c, lm.q, true, dx);
        store_slots<M, FULL, CM>(gy + row * W, L, lm.c, lm.q, true, dy);
      }
    };
  };
  if (weights_in_smem) {
    uint64_t* wbar = reinterpret_cast<uint64_t*>(smem) + 2 * kMaxStages;
    float4* wsm = reinterpret_cast<float4*>(smem + kBarrierBytes);
    if (threadIdx.x == 0) {
      mbar_init(wbar, 1);
      fence_mbarrier_init();
      mbar_arrive_expect_tx(wbar, static_cast<uint32_t>(wbytes));
      bulk_g2s(wsm, ws, static_cast<uint32_t>(wbytes), wbar);
    }
    __syncthreads();
    if (!mbar_wait(wbar, 0, 4)) return;
    const SharedChunks chunks{static_cast<uint32_t>(__cvta_generic_to_shared(wsm + t)),
                              T * static_cast<int>(sizeof(float4))};
    // stages follow the weights
    staged_loop<3, true>(smem, smem + wbytes, stages, R, rows, W, src, body(chunks));
  } else {
    const GlobalChunks chunks{ws + t, T};
    staged_loop<3, true>(smem, smem, stages, R, rows, W, src, body(chunks));
  }
  if (lm.active) {
    const int64_t slot = static_cast<int64_t>(blockIdx.x) * R + r;
    store_partial<M, FULL>(partial + slot * numel, L, mags, lm.c, lm.q, acc);
  }
}

// Staged backward over row pairs: a stage holds 2 R rows per operand and each warp
// carries rows 2 r and 2 r + 1 of it through row_vjp2 (paired f32x2 arithmetic).  dx and
// dy of each row equal those of tp_backward_staged bit for bit; the weight-gradient slot
// takes the two rows' terms path by path (another float32 summation order).  A missing
// second row (odd row count) computes on zeros and stores nothing.
template <int M, bool FULL, bool CM = false>
__global__ void __launch_bounds__(kStagedWarps * 32, 1)
    tp_backward_paired(const float* __restrict__ x, const float* __restrict__ y,
                       const float4* __restrict__ ws, const float* __restrict__ go,
                       float* __restrict__ gx, float* __restrict__ gy,
                       float* __restrict__ partial, int64_t numel, int64_t rows, TpLayout L,
                       Mags mags, int groups, int R, int stages, int weights_in_smem) {
  extern __shared__ __align__(128) unsigned char smem[];
  using P = Paths<M, FULL>;
  constexpr int S = 2 * M + 2;
  const int warp = threadIdx.x >> 5;
  const int r = warp / groups;
  const int T = groups * 32;
  const int t = (warp % groups) * 32 + (threadIdx.x & 31);
  const LaneMap<FULL> lm(warp % groups, threadIdx.x & 31, L.C);
  const size_t wbytes = static_cast<size_t>(P::chunks) * T * sizeof(float4);
  const int RB = 2 * R;  // rows per stage block
  float acc[P::n];
#pragma unroll
  for (int i = 0; i < P::n; ++i) acc[i] = 0.0f;
  const float* src[3] = {x, y, go};
  const int64_t W = L.width;
  auto body = [&](const auto& chunks) {
    return [&](const float* stage, int64_t row) {
      const bool two = row + 1 < rows;
      float2 a[S], b[S], g[S], dx[S], dy[S];
      auto load_pair = [&](const float* base, float2 (&v)[S]) {
        float u0[S], u1[S];
        load_slots<M, FULL, CM>(SharedRow(base), L, lm.c, lm.q, u0);
        load_slots<M, FULL, CM>(SharedRow(base + W), L, lm.c, lm.q, u1);
#pragma unroll
        for (int k = 0; k < S; ++k) v[k] = make_float2(u0[k], two ? u1[k] : 0.f);
      };
      load_pair(stage, a);
      load_pair(stage + RB * W, b);
      load_pair(stage + 2 * RB * W, g);
      row_vjp2<M, FULL>(a, b, g, chunks, lm.q, dx, dy, acc);
      if (lm.active) {
        auto store_pair = [&](float* dst, const float2 (&v)[S]) {
          float v0[S], v1[S];
#pragma unroll
          for (int k = 0; k < S; ++k) {
            v0[k] = v[k].x;
            v1[k] = v[k].y;
          }
          store_slots<M, FULL, CM>(dst + row * W, L, lm.c, lm.q, true, v0);
          if (two) store_slots<M, FULL, CM>(dst + (row + 1) * W, L, lm.c, lm.q, true, v1);
        };
        store_pair(gx, dx);
        store_pair(gy, dy);
      }
    };
  };
  if (weights_in_smem) {
    uint64_t* wbar = reinterpret_cast<uint64_t*>(smem) + 2 * kMaxStages;
    float4* wsm = reinterpret_cast<float4*>(smem + kBarrierBytes);
    if (threadIdx.x == 0) {
      mbar_init(wbar, 1);
      fence_mbarrier_init();
      mbar_arrive_expect_tx(wbar, static_cast<uint32_t>(wbytes));
      bulk_g2s(wsm, ws, static_cast<uint32_t>(wbytes), wbar);
    }
    __syncthreads();
    if (!mbar_wait(wbar, 0, 4)) return;
    const SharedChunks chunks{static_cast<uint32_t>(__cvta_generic_to_shared(wsm + t)),
                              T * static_cast<int>(sizeof(float4))};
    staged_loop<3, true, 2>(smem, smem + wbytes, stages, R, rows, W, src, body(chunks));
  } else {
    const GlobalChunks chunks{ws + t, T};
    staged_loop<3, true, 2>(smem, smem, stages, R, rows, W, src, body(chunks));
  }
  if (lm.active) {
    const int64_t slot = static_cast<int64_t>(blockIdx.x) * R + r;
    store_partial<M, FULL>(partial + slot * numel, L, mags, lm.c, lm.q, acc);
  }
}

// ------------------------------------------------------------ channel-tiled backward
//
// For channel counts whose warps do not fill a staged CTA (full parity: C = 96
// gives 6 warps, C = 256 needs 16 channel groups), the CTA works on a tile of Ct
// channels of every row instead: the tile's slice of a row arrives by two tiled
// TMA boxes per operand (tmap.cuh) and lands as a row of a Ct-channel product,
// so the per-row arithmetic is that of the untiled kernel.  CTA b serves tile
// b % ntiles and the blocks of R rows (b / ntiles) + k * (grid / ntiles); slot
// (b / ntiles) * R + r of the weight-gradient partials holds the tile's channels,
// the other tiles' CTAs of the same slot index the rest, so every partial row is
// written in full.

template <int M, bool FULL, bool CM = false>
__global__ void __launch_bounds__(kStagedWarps * 32, 1)
    tp_backward_tiled(const __grid_constant__ RowTileMaps maps, const float4* __restrict__ ws,
                      float* __restrict__ gx, float* __restrict__ gy,
                      float* __restrict__ partial, int64_t numel, int64_t rows, TpLayout L,
                      TpLayout Lt, Mags mags, int gt, int R, int stages, int ntiles,
                      int weights_in_smem) {
  extern __shared__ __align__(128) unsigned char smem[];
  using P = Paths<M, FULL>;
  constexpr int S = 2 * M + 2;
  constexpr int S0 = FULL ? 2 : 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = static_cast<int>(blockIdx.x % ntiles);
  const int64_t cta = blockIdx.x / ntiles, ctas = gridDim.x / ntiles;
  const int r = warp / gt;
  const int Ct = Lt.C, c0 = tile * Ct;
  const int Tt = gt * 32;                       // threads of one row slot of the tile
  const int T = ntiles * Tt;                    // threads of all channel groups
  const int tl = (warp % gt) * 32 + lane;       // thread within the tile's row slot
  const LaneMap<FULL> lm(tile * gt + warp % gt, lane, L.C);
  const int cl = lm.active ? lm.c - c0 : 0;     // channel within the tile
  const int64_t Wt = Lt.width;
  const size_t wbytes = weights_in_smem ? static_cast<size_t>(P::chunks) * Tt * sizeof(float4)
                                        : 0;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  unsigned* done = reinterpret_cast<unsigned*>(full + kMaxStages);
  uint64_t* wbar = full + 2 * kMaxStages;
  float4* wsm = reinterpret_cast<float4*>(smem + kBarrierBytes);
  float* buf = reinterpret_cast<float*>(smem + kBarrierBytes + wbytes);
  const int64_t nblocks = (rows + R - 1) / R;
  const uint32_t scalar_bytes = static_cast<uint32_t>(S0 * Ct * 4);

  // stage s <- rows of block b of this tile: two boxes per operand row
  auto issue = [&](int s, int64_t b) {
    const int64_t row0 = b * R;
    const int nr = rows - row0 < R ? static_cast<int>(rows - row0) : R;
    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(3 * nr * Wt * 4));
    float* st = buf + static_cast<int64_t>(s) * 3 * R * Wt;
    for (int t = 0; t < 3; ++t) {
      for (int rr = 0; rr < nr; ++rr) {
        float* dst = st + (t * R + rr) * Wt;
        const int z = static_cast<int>(row0 + rr);
        tma_load_3d(dst, &maps.m[2 * t], c0, 0, z, &full[s]);
        if constexpr (M > 0) {
          tma_load_3d(reinterpret_cast<unsigned char*>(dst) + scalar_bytes, &maps.m[2 * t + 1],
                      CM ? c0 : 2 * c0, 0, z, &full[s]);
        }
      }
    }
  };

  if (threadIdx.x == 0) {
    for (int st = 0; st < stages; ++st) {
      mbar_init(&full[st], 1);
      done[st] = 0;
    }
    if (weights_in_smem) mbar_init(wbar, 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (weights_in_smem) {
      // chunk k of the tile's threads: ws[k * T + tile * Tt .. + Tt)
      mbar_arrive_expect_tx(wbar, static_cast<uint32_t>(wbytes));
      for (int k = 0; k < P::chunks; ++k)
        bulk_g2s(wsm + k * Tt, ws + static_cast<int64_t>(k) * T + tile * Tt,
                 static_cast<uint32_t>(Tt * sizeof(float4)), wbar);
    }
    for (int st = 0; st < stages; ++st) {
      const int64_t b = cta + st * ctas;
      if (b < nblocks) issue(st, b);
    }
  }
  float acc[P::n];
#pragma unroll
  for (int i = 0; i < P::n; ++i) acc[i] = 0.0f;
  bool ok = true;
  auto run = [&](const auto& chunks) {
    int s = 0;
    uint32_t round = 0;
    const int nwarps = blockDim.x >> 5;
    for (int64_t b = cta; b < nblocks && ok; b += ctas) {
      ok = mbar_wait(&full[s], round & 1, 1);
      if (!ok) break;
      const int64_t row = b * R + r;
      if (row < rows) {
        const float* st = buf + static_cast<int64_t>(s) * 3 * R * Wt + r * Wt;
        float a[S], bb[S], g[S], dx[S], dy[S];
        load_slots<M, FULL, CM>(SharedRow(st), Lt, cl, lm.q, a);
        load_slots<M, FULL, CM>(SharedRow(st + R * Wt), Lt, cl, lm.q, bb);
        load_slots<M, FULL, CM>(SharedRow(st + 2 * R * Wt), Lt, cl, lm.q, g);
        row_vjp<M, FULL>(a, bb, g, chunks, lm.q, dx, dy, acc);
        if (lm.active) {
          store_slots<M, FULL, CM>(gx + row * L.width, L, lm.c, lm.q, true, dx);
          store_slots<M, FULL, CM>(gy + row * L.width, L, lm.c, lm.q, true, dy);
        }
      }
      __syncwarp();
      if (lane == 0) {
        unsigned prev;
        asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "r"(smem_addr(&done[s]))
                     : "memory");
        if (prev + 1 == static_cast<unsigned>(nwarps) * (round + 1)) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          const int64_t next = b + static_cast<int64_t>(stages) * ctas;
          if (next < nblocks) issue(s, next);
        }
      }
      if (++s == stages) {
        s = 0;
        ++round;
      }
    }
  };
  if (weights_in_smem) {
    ok = mbar_wait(wbar, 0, 4);
    if (ok)
      run(SharedChunks{static_cast<uint32_t>(__cvta_generic_to_shared(wsm + tl)),
                       Tt * static_cast<int>(sizeof(float4))});
  } else {
    run(GlobalChunks{ws + tile * Tt + tl, T});
  }
  if (!ok) {
    if (threadIdx.x == 0) {
      // a wait ran out: let copies already issued land before the CTA exits
      for (int st = 0; st < stages; ++st) mbar_wait(&full[st], 0, 3, kDrainLimitNs);
    }
    return;
  }
  if (lm.active) {
    const int64_t slot = cta * R + r;
    store_partial<M, FULL>(partial + slot * numel, L, mags, lm.c, lm.q, acc);
  }
}

// ------------------------------------------------------------ small kernels

// Magnitude-scaled weights in the per-thread order of row_vjp: chunk k of thread
// t (channel group t / 32, lane t % 32) holds the weights of paths vjp[4k..4k+3]
// for that lane's (channel, world), at ws[k * T + t]; unused entries are zero.
// blockIdx.y is the chunk, so the chunks are written by as many CTAs in parallel
// (one CTA writing every chunk took 9 us at TP(128, 6, full)).
template <int M, bool FULL, bool CM = false>
__global__ void prescale_kernel(const float* __restrict__ w, float4* __restrict__ ws,
                                TpLayout L, Mags mags, int groups) {
  using P = Paths<M, FULL>;
  const int T = groups * 32;
  const int chunk = blockIdx.y;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
    const LaneMap<FULL> lm(t / 32, t % 32, L.C);
    static_for<P::chunks>([&](auto k) {
      if (k != chunk) return;
      float v[4];
      static_for<4>([&](auto e) {
        constexpr int pos = 4 * k + e;
        if constexpr (pos < P::n) {
          constexpr int I = P::vjp.idx[pos];
          constexpr ChanPath cp = P::table.p[I];
          const bool used = lm.active && (!FULL || cp.copied || lm.q == 0);
          v[e] = used ? w[weight_index<M, FULL, I>(L.C, lm.c, lm.q)] * mags.m[cp.cls] : 0.0f;
        } else {
          v[e] = 0.0f;
        }
      });
      ws[k * T + t] = make_float4(v[0], v[1], v[2], v[3]);
    });
  }
}

// dw[i] = sum over slots of partial[slot][i], in a fixed order: thread (r, col)
// sums slots r, r + 8, ... and the 8 partial sums are added in order r = 0..7.
__global__ void __launch_bounds__(256)
    reduce_slots_kernel(const float* __restrict__ partial, float* __restrict__ dst,
                        int64_t numel, int64_t slots) {
  __shared__ float buf[8][33];
  const int col = threadIdx.x & 31;
  const int r = threadIdx.x >> 5;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 32 + col;
  float s = 0.0f;
  if (i < numel) {
    for (int64_t k = r; k < slots; k += 8) s += partial[k * numel + i];
  }
  buf[r][col] = s;
  __syncthreads();
  if (r == 0 && i < numel) {
    float t = buf[0][col];
#pragma unroll
    for (int k = 1; k < 8; ++k) t += buf[k][col];
    dst[i] = t;
  }
}

__global__ void zero_kernel(float* __restrict__ dst, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = 0.0f;
}

// ------------------------------------------------------------------ dispatch

using ForwardDirectFn = void (*)(const float*, const float*, const float*, float*, int64_t,
                                 TpLayout, Mags, int, int64_t, int64_t, bool);
using BackwardDirectFn = void (*)(const float*, const float*, const float4*, const float*,
                                  float*, float*, float*, int64_t, int64_t, TpLayout, Mags, int,
                                  int64_t, int64_t, bool);
using ForwardStagedFn = void (*)(const float*, const float*, const float*, float*, int64_t,
                                 TpLayout, Mags, int, int, int);
using BackwardStagedFn = void (*)(const float*, const float*, const float4*, const float*,
                                  float*, float*, float*, int64_t, int64_t, TpLayout, Mags, int,
                                  int, int, int);
using PrescaleFn = void (*)(const float*, float4*, TpLayout, Mags, int);
using ForwardGroupedFn = void (*)(const float*, const float*, const float*, float*, int64_t,
                                  TpLayout, Mags, int, int64_t, bool);
using BackwardTiledFn = void (*)(RowTileMaps, const float4*, float*, float*, float*, int64_t,
                                 int64_t, TpLayout, TpLayout, Mags, int, int, int, int, int);

// ICTC_ONLY_ORDER=m builds one order only (quick register/spill checks).
#ifdef ICTC_ONLY_ORDER
constexpr bool compiled_order(int m) { return m == ICTC_ONLY_ORDER; }
#else
constexpr bool compiled_order(int) { return true; }
#endif

struct Kernels {
  ForwardStagedFn fwd_wide;  // null when the weights do not fit in shared memory
  ForwardDirectFn fwd_direct;
  BackwardDirectFn bwd_direct;
  ForwardStagedFn fwd_staged;
  BackwardStagedFn bwd_staged;
  PrescaleFn prescale;
  int chunks;  // float4 weight chunks per thread (Paths::chunks)
  ForwardGroupedFn fwd_grouped;
  BackwardTiledFn bwd_tiled;
  BackwardStagedFn bwd_paired;  // row pairs through paired f32x2 arithmetic, or null
  ForwardStagedFn fwd_wide_paired;  // null when the weights do not fit in shared memory
};

// Row-paired backward where the sweep measured it faster than the scalar staged kernel:
// full parity, m_max 3 and 4 (backward 1.11-1.22x at C = 32-128; at m_max 5-6 the
// paired per-row state spills at 255 registers and it lost 0.81-0.93x, and below 3 two
// scalar CTAs per SM win).  Both layouts, so they stay bit-identical to each other.
template <int M, bool FULL, bool CM>
constexpr BackwardStagedFn paired_for() {
  if constexpr (FULL && (M == 3 || M == 4)) return &tp_backward_paired<M, FULL, CM>;
  else return nullptr;
}

// Kernels of one (order, parity, frequency-block layout); the layout is a template
// parameter so that each layout runs its own straight-line slot accesses.
template <int M, bool FULL, bool CM>
constexpr Kernels kernels_for() {
  if constexpr (compiled_order(M)) {
    ForwardStagedFn wide = nullptr;
    if constexpr (wide_forward_fits<M, FULL>()) wide = &tp_forward_wide<M, FULL, CM>;
    return Kernels{wide, &tp_forward_direct<M, FULL, CM>, &tp_backward_direct<M, FULL, CM>,
                   &tp_forward_staged<M, FULL, CM>, &tp_backward_staged<M, FULL, CM>,
                   &prescale_kernel<M, FULL>, Paths<M, FULL>::chunks,
                   &tp_forward_grouped<M, FULL, CM>, &tp_backward_tiled<M, FULL, CM>,
                   paired_for<M, FULL, CM>(),
                   wide == nullptr ? nullptr : &tp_forward_wide_paired<M, FULL, CM>};
  } else {
    return Kernels{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0, nullptr, nullptr,
                   nullptr, nullptr};
  }
}

template <int... Ms>
constexpr auto make_table(std::integer_sequence<int, Ms...>) {
  struct T { Kernels k[2][2][sizeof...(Ms)]; };  // [layout][full][m_max]
  return T{{{{kernels_for<Ms, false, false>()...}, {kernels_for<Ms, true, false>()...}},
            {{kernels_for<Ms, false, true>()...}, {kernels_for<Ms, true, true>()...}}}};
}

const auto kKernels = make_table(std::make_integer_sequence<int, kMaxOrder + 1>{});

int validate(int64_t rows, int32_t channels, int32_t m_max, int32_t parity,
             int32_t normalization) {
  if (rows < 0) return fail(ICTC_ERR_INVALID, "rows must be >= 0 (got %lld)", (long long)rows);
  if (channels < 1) return fail(ICTC_ERR_INVALID, "channels must be >= 1 (got %d)", channels);
  if (m_max < 0) return fail(ICTC_ERR_INVALID, "m_max must be >= 0 (got %d)", m_max);
  if (parity != ICTC_PARITY_CANONICAL && parity != ICTC_PARITY_FULL)
    return fail(ICTC_ERR_INVALID, "parity must be 0 (canonical) or 1 (full), got %d", parity);
  if (normalization != ICTC_NORM_COMPONENT && normalization != ICTC_NORM_NORM)
    return fail(ICTC_ERR_INVALID, "normalization must be 0 (component) or 1 (norm), got %d",
                normalization);
  if (m_max > kMaxOrder)
    return fail(ICTC_ERR_UNSUPPORTED, "m_max=%d exceeds the compiled maximum %d", m_max,
                kMaxOrder);
  const TpLayout L = tp_layout(channels, m_max, parity == ICTC_PARITY_FULL);
  if (L.width > (int64_t(1) << 30))
    return fail(ICTC_ERR_UNSUPPORTED, "row width %lld too large", (long long)L.width);
  return ICTC_OK;
}

int64_t weight_numel(int C, int m_max, bool full) {
  return static_cast<int64_t>(build_table(m_max, full).units) * C;
}

int current_device(int* device) {
  const cudaError_t e = cudaGetDevice(device);
  return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "cudaGetDevice");
}

// Direct grid: a multiple of `groups` warps so that every warp keeps one channel
// group; `slots` warps share each group and split the rows round-robin.
struct DirectPlan {
  int groups;
  int64_t slots, nwarps, blocks;
};

int plan_direct(const void* kernel, int device, int64_t rows, int C, bool full, DirectPlan* out) {
  int per_sm = 0;
  const cudaError_t e =
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kDirectThreads, 0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  out->groups = static_cast<int>(ceil_div(C, full ? 16 : 32));
  const int64_t resident =
      static_cast<int64_t>(sm_count(device)) * (per_sm > 0 ? per_sm : 1) * (kDirectThreads / 32);
  int64_t slots = resident / out->groups;
  if (slots < 1) slots = 1;
  if (slots > rows) slots = rows > 0 ? rows : 1;
  out->slots = slots;
  out->nwarps = slots * out->groups;
  out->blocks = ceil_div(out->nwarps * 32, kDirectThreads);
  return ICTC_OK;
}

// Staged grid: one persistent CTA per SM of R * groups warps (R rows per stage).
// With `weight_bytes` > 0 the weights go to shared memory in front of the stages
// when at least three stages still fit.
struct StagedPlan {
  bool ok, weights_in_smem, paired;
  int groups, R, warps, stages;
  int64_t grid;
  size_t smem;
};

// ctas_per_sm > 1: the stage ring shares the SM's shared memory with that many CTAs
// (the caller checks that their registers fit), and the grid has that many per SM.
StagedPlan plan_staged(int device, int64_t rows, const TpLayout& L, bool full, int tensors,
                       size_t weight_bytes, int max_warps = kStagedWarps, int max_stages = kMaxStages,
                       bool weights_required = false, int ctas_per_sm = 1, int rows_per_warp = 1) {
  StagedPlan p{};
  // per-SM shared memory of sm_100 (228 KB) less the 1 KB each CTA reserves, and a margin
  const size_t budget =
      ctas_per_sm > 1 ? (228 * 1024) / static_cast<size_t>(ctas_per_sm) - 2 * 1024
                      : kStagedSmemBudget;
  p.groups = static_cast<int>(ceil_div(L.C, full ? 16 : 32));
  if (p.groups > max_warps || L.width % 4 != 0 || rows == 0) return p;
  p.R = max_warps / p.groups;
  p.warps = p.R * p.groups;
  const size_t stage_bytes =
      static_cast<size_t>(tensors) * p.R * rows_per_warp * L.width * sizeof(float);
  if (weight_bytes > 0 && budget > kBarrierBytes + weight_bytes) {
    const int fit =
        static_cast<int>((budget - kBarrierBytes - weight_bytes) / stage_bytes);
    if (fit >= (weights_required ? 2 : 3)) {
      p.weights_in_smem = true;
      p.stages = fit < max_stages ? fit : max_stages;
      p.smem = kBarrierBytes + weight_bytes + static_cast<size_t>(p.stages) * stage_bytes;
    }
  }
  if (!p.weights_in_smem) {
    if (weights_required) return p;
    const int fit = static_cast<int>((budget - kBarrierBytes) / stage_bytes);
    p.stages = fit < kMaxStages ? fit : kMaxStages;
    if (p.stages < 2) return p;
    p.smem = kBarrierBytes + static_cast<size_t>(p.stages) * stage_bytes;
  }
  const int64_t nblocks = ceil_div(rows, static_cast<int64_t>(p.R) * rows_per_warp);
  p.grid = static_cast<int64_t>(sm_count(device)) * ctas_per_sm;
  if (p.grid > nblocks) p.grid = nblocks;
  p.ok = true;
  return p;
}

// Channel-tiled backward (tp_backward_tiled): used where the untiled staged CTA
// cannot be formed (more than kStagedWarps channel groups, e.g. C = 256 full) and
// rows are long enough (m_max >= 3).  Measured over the benchmark sweep (65,536
// rows, fraction of HBM): C = 256 full m_max 3-6 backward 0.70-0.74 against the
// direct kernel's 0.40-0.54, but m_max 1-2 0.42 / 0.60 against 0.69 / 0.67, and a
// 32-channel tiling of C = 96 full lost to the 6-warp untiled CTA at every m_max
// below 6, so those keep the untiled kernels.  Tiles of Ct channels (Ct in 128,
// 64, 32, 16, a multiple of the channels per warp, dividing C) with gt = Ct /
// channels-per-warp groups and R = 8 / gt rows per stage; floor(SMs / ntiles)
// CTAs per tile, so every tile has as many CTAs.
struct TiledPlan {
  bool ok, weights_in_smem;
  int Ct, gt, R, ntiles, stages;
  int64_t ctas, grid;
  size_t smem;
};

TiledPlan plan_tiled(int device, int64_t rows, const TpLayout& L, bool full, int chunks) {
  TiledPlan p{};
  const int cpw = full ? 16 : 32;
  const int groups = static_cast<int>(ceil_div(L.C, cpw));
  const int m_max = static_cast<int>((L.width / L.C / (full ? 2 : 1) - 1) / 2);
  if (groups <= kStagedWarps || m_max < 3 || rows == 0 || rows > INT32_MAX || L.C % 16 != 0)
    return p;
  for (int ct : {128, 64, 32, 16}) {
    if (ct % cpw == 0 && ct < L.C && L.C % ct == 0) {
      p.Ct = ct;
      break;
    }
  }
  if (p.Ct == 0) return p;
  p.gt = p.Ct / cpw;
  p.R = kStagedWarps / p.gt;
  p.ntiles = L.C / p.Ct;
  const TpLayout Lt = tp_layout(p.Ct, m_max, full, L.cm);
  const size_t stage_bytes = static_cast<size_t>(3) * p.R * Lt.width * sizeof(float);
  const size_t wbytes = static_cast<size_t>(chunks) * p.gt * 32 * sizeof(float4);
  if (kStagedSmemBudget > kBarrierBytes + wbytes) {
    const int fit = static_cast<int>((kStagedSmemBudget - kBarrierBytes - wbytes) / stage_bytes);
    if (fit >= 3) {
      p.weights_in_smem = true;
      p.stages = fit < kMaxStages ? fit : kMaxStages;
      p.smem = kBarrierBytes + wbytes + static_cast<size_t>(p.stages) * stage_bytes;
    }
  }
  if (!p.weights_in_smem) {
    const int fit = static_cast<int>((kStagedSmemBudget - kBarrierBytes) / stage_bytes);
    p.stages = fit < kMaxStages ? fit : kMaxStages;
    if (p.stages < 2) return p;
    p.smem = kBarrierBytes + static_cast<size_t>(p.stages) * stage_bytes;
  }
  const int64_t nblocks = ceil_div(rows, p.R);
  p.ctas = sm_count(device) / p.ntiles;
  if (p.ctas < 1) p.ctas = 1;
  if (p.ctas > nblocks) p.ctas = nblocks;
  p.grid = p.ctas * p.ntiles;
  p.ok = true;
  return p;
}

bool aligned16(std::initializer_list<const void*> ptrs) {
  for (const void* p : ptrs)
    if (!aligned(p, 16)) return false;
  return true;
}

// Two staged backward CTAs per SM where registers allow (default);
// ICTC_TP_BACKWARD_PAIRS=0 keeps one (tests cover both).
bool staged_pairs_enabled() {
  const char* v = getenv("ICTC_TP_BACKWARD_PAIRS");
  return v == nullptr || strcmp(v, "0") != 0;
}

// Row-paired backward where compiled (default); ICTC_TP_BACKWARD_ROWPAIR=0 runs the
// scalar staged kernel instead (tests cover both).
bool row_pairs_enabled() {
  const char* v = getenv("ICTC_TP_BACKWARD_ROWPAIR");
  return v == nullptr || strcmp(v, "0") != 0;
}

// Backward workspace: [per-thread float4 weight chunks][slots x numel partials].
size_t weight_chunk_bytes(const Kernels& k, int C, bool full) {
  const int64_t T = ceil_div(C, full ? 16 : 32) * 32;
  return static_cast<size_t>(k.chunks) * static_cast<size_t>(T) * sizeof(float4);
}

// CTAs of `warps` warps of kernel fn whose registers fit one SM together (at most 2).
int ctas_by_registers(const void* fn, int warps) {
  static std::mutex mu;
  static const void* seen[64] = {};
  static int regs_of[64] = {};
  int regs = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    int slot = -1;
    for (int i = 0; i < 64; ++i) {
      if (seen[i] == fn) {
        regs = regs_of[i];
        break;
      }
      if (seen[i] == nullptr) {
        slot = i;
        break;
      }
    }
    if (regs == 0) {
      cudaFuncAttributes a{};
      if (cudaFuncGetAttributes(&a, fn) != cudaSuccess) {
        cudaGetLastError();
        return 1;
      }
      regs = a.numRegs;
      if (slot >= 0) {
        seen[slot] = fn;
        regs_of[slot] = regs;
      }
    }
  }
  const int per_cta = ((regs + 7) / 8) * 8 * warps * 32;  // allocation in 8-register steps
  const int n = per_cta > 0 ? 65536 / per_cta : 1;
  return n < 1 ? 1 : (n > 2 ? 2 : n);  // three per SM measured slower (sweep 0.740 vs 0.748)
}

// Plan of the staged backward: where the kernel's registers let two CTAs share an SM
// (small orders: m_max <= 2 full, <= 3 canonical, m_max 3 full at C = 96), each gets half
// the shared memory for its stage ring and the grid doubles, so twice the warps hide the
// per-row latencies of those short rows.  Measured over the benchmark sweep (backward
// time, one CTA per SM / two): full parity 1.13-1.63x at every such shape; canonical
// 1.03-1.34x where the single CTA has fewer than 8 warps (C = 96) or m_max = 1 at
// C >= 64, but 0.79-0.92x at m_max 2-3 otherwise (their single CTA already reaches
// 0.8-0.98 of HBM at 65,536 rows) and 0.84x at C = 32, m_max 1; those keep one CTA.
// Where one CTA per SM remains and a row-paired kernel is compiled (full parity, m_max
// 3-4), each warp takes two rows at a time (stages of 2 R rows).
StagedPlan plan_staged_backward(int device, const Kernels& k, int64_t rows, const TpLayout& L,
                                bool full) {
  const size_t wb = weight_chunk_bytes(k, L.C, full);
  const StagedPlan p = plan_staged(device, rows, L, full, 3, wb);
  if (!p.ok) return p;
  const int m_max = static_cast<int>((L.width - L.fbase) / L.fstride);
  const int ctas = !staged_pairs_enabled() ||
                           (!full && p.warps >= kStagedWarps && !(m_max == 1 && L.C >= 64))
                       ? 1
                       : ctas_by_registers(reinterpret_cast<const void*>(k.bwd_staged), p.warps);
  if (ctas > 1) {
    const StagedPlan q =
        plan_staged(device, rows, L, full, 3, wb, kStagedWarps, kMaxStages, false, ctas);
    if (q.ok) return q;
  }
  if (k.bwd_paired != nullptr && row_pairs_enabled()) {
    // two rows per warp: stages of 2 R rows
    StagedPlan q =
        plan_staged(device, rows, L, full, 3, wb, kStagedWarps, kMaxStages, false, 1, 2);
    if (q.ok) {
      q.paired = true;
      return q;
    }
  }
  return p;
}

int64_t backward_slots(int device, const Kernels& k, int64_t rows, const TpLayout& L, bool full,
                       int* status) {
  DirectPlan d{};
  *status = plan_direct(reinterpret_cast<const void*>(k.bwd_direct), device, rows, L.C, full, &d);
  const StagedPlan s = plan_staged_backward(device, k, rows, L, full);
  int64_t slots = d.slots;
  if (s.ok && s.grid * s.R > slots) slots = s.grid * s.R;
  const TiledPlan t = plan_tiled(device, rows, L, full, k.chunks);
  if (t.ok && t.ctas * t.R > slots) slots = t.ctas * t.R;
  return slots;
}

}  // namespace

int tp_take_device_error(int* code) {
  cudaError_t e;
  if (take_unit_device_error(code, &e) != 0) return cuda_fail(e, "TensorProduct device error flag");
  return ICTC_OK;
}

}  // namespace ictc

using namespace ictc;

extern "C" int32_t ictc_o2_tp_weight_numel(int32_t channels, int32_t m_max, int32_t parity,
                                           int64_t* numel) {
  if (numel == nullptr) return fail(ICTC_ERR_INVALID, "numel is null");
  const int st = validate(0, channels, m_max, parity, ICTC_NORM_COMPONENT);
  if (st != ICTC_OK) return st;
  *numel = weight_numel(channels, m_max, parity == ICTC_PARITY_FULL);
  return ICTC_OK;
}

extern "C" int32_t ictc_o2_tp_path_table(int32_t m_max, int32_t parity, int32_t* table,
                                         int32_t capacity_paths, int32_t* count) {
  if (count == nullptr) return fail(ICTC_ERR_INVALID, "count is null");
  const int st = validate(0, 1, m_max, parity, ICTC_NORM_COMPONENT);
  if (st != ICTC_OK) return st;
  const PathTable t = build_table(m_max, parity == ICTC_PARITY_FULL);
  *count = t.n;
  if (table == nullptr) return ICTC_OK;
  if (capacity_paths < t.n)
    return fail(ICTC_ERR_INVALID, "table holds %d paths, need %d", capacity_paths, t.n);
  for (int p = 0; p < t.n; ++p) {
    int32_t* r = table + p * 23;
    const ChanPath& c = t.p[p];
    r[0] = c.in1; r[1] = c.in2; r[2] = c.out; r[3] = c.cls; r[4] = c.unit; r[5] = c.copied;
    r[6] = c.nt;
    for (int k = 0; k < 4; ++k) {
      r[7 + 4 * k] = k < c.nt ? c.t[k].i : 0;
      r[8 + 4 * k] = k < c.nt ? c.t[k].j : 0;
      r[9 + 4 * k] = k < c.nt ? c.t[k].k : 0;
      r[10 + 4 * k] = k < c.nt ? c.t[k].s : 0;
    }
  }
  return ICTC_OK;
}

namespace {

int32_t tp_forward_impl(const float* left, const float* right, const float* weight,
                        float* output, int64_t rows, int32_t channels, int32_t m_max,
                        int32_t parity, int32_t normalization, int32_t layout, void* stream) {
  int st = validate(rows, channels, m_max, parity, normalization);
  if (st != ICTC_OK) return st;
  if (layout != ICTC_LAYOUT_CHANNEL_MAJOR && layout != ICTC_LAYOUT_COMPONENT_MAJOR)
    return fail(ICTC_ERR_INVALID, "layout must be ICTC_LAYOUT_CHANNEL_MAJOR or _COMPONENT_MAJOR");
  if (rows == 0) return ICTC_OK;
  if (!left || !right || !weight || !output)
    return fail(ICTC_ERR_INVALID, "null tensor pointer");
  if (!aligned(left, 4) || !aligned(right, 4) || !aligned(weight, 4) || !aligned(output, 4))
    return fail(ICTC_ERR_INVALID, "tensor pointers must be 4-byte aligned");
  const bool full = parity == ICTC_PARITY_FULL;
  const TpLayout L = tp_layout(channels, m_max, full, layout);
  const Kernels& k = kKernels.k[L.cm][full ? 1 : 0][m_max];
  const Mags mags = tp_mags(normalization);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int device = 0;
  if ((st = current_device(&device)) != ICTC_OK) return st;
  const char* variant = getenv("ICTC_TP_FORWARD");
  const bool al16 = aligned16({left, right, output});
  // Default: the wide staged kernel (16 warps, weights and two-row stages in shared
  // memory) from m_max = 4 up, where its rows are long enough to keep the bulk
  // copies busy; below that, and when it does not fit, the grouped kernel.
  // Measured over the benchmark sweep (C 32..256, m_max 1..6, both parities).
  // Row-paired wide forward by default at full parity from m_max = 4 up where its
  // 8-warp CTA is full (channel groups dividing 8): measured at 65,536 rows after an
  // L2 flush, C = 128 full m_max 6 / 5 / 4 0.470 -> 0.418 / 0.388 -> 0.361 / 0.321 ->
  // 0.311 ms, C = 64 and 32 full m_max 6 0.243 -> 0.218 and 0.130 -> 0.118 ms; it lost
  // at C = 96 full (six groups: 0.373 -> 0.375 ms) and at canonical parity (C = 128
  // m_max 6: 0.202 -> 0.212 ms), which keep the wide kernel.
  const int fwd_groups = static_cast<int>(ceil_div(channels, full ? 16 : 32));
  const bool want_pair =
      (variant == nullptr && full && m_max >= 4 && kWidePairWarps % fwd_groups == 0) ||
      (variant != nullptr && strcmp(variant, "widepair") == 0);
  const StagedPlan pp =
      (want_pair && k.fwd_wide_paired && al16)
          ? plan_staged(device, rows, L, full, 2, weight_chunk_bytes(k, channels, full),
                        kWidePairWarps, 2, true, 1, 2)
          : StagedPlan{};
  if (pp.ok) {
    if ((st = allow_smem(reinterpret_cast<const void*>(k.fwd_wide_paired), pp.smem)) != ICTC_OK)
      return st;
    k.fwd_wide_paired<<<static_cast<unsigned>(pp.grid), pp.warps * 32, pp.smem, s>>>(
        left, right, weight, output, rows, L, mags, pp.groups, pp.R, pp.stages);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "tp_forward launch");
  }
  const bool want_wide = (variant == nullptr && m_max >= 4) ||
                         (variant != nullptr &&
                          (strcmp(variant, "wide") == 0 || want_pair));  // also the fallback
  const StagedPlan wp =
      (want_wide && k.fwd_wide && al16)
          ? plan_staged(device, rows, L, full, 2, weight_chunk_bytes(k, channels, full),
                        kWideWarps, 2, true)
          : StagedPlan{};
  if (wp.ok) {
    if ((st = allow_smem(reinterpret_cast<const void*>(k.fwd_wide), wp.smem)) != ICTC_OK)
      return st;
    k.fwd_wide<<<static_cast<unsigned>(wp.grid), wp.warps * 32, wp.smem, s>>>(
        left, right, weight, output, rows, L, mags, wp.groups, wp.R, wp.stages);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "tp_forward launch");
  }
  if (variant == nullptr || strcmp(variant, "grouped") == 0 || want_wide) {
    const bool vec2 = (L.width % 2 == 0) && aligned(left, 8) && aligned(right, 8) &&
                      aligned(output, 8);
    const int groups = static_cast<int>(ceil_div(channels, full ? 16 : 32));
    const size_t smem = static_cast<size_t>(k.chunks) * 32 * sizeof(float4);
    const void* fn = reinterpret_cast<const void*>(k.fwd_grouped);
    if ((st = allow_smem(fn, smem)) != ICTC_OK) return st;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn,
                                                                  kGroupFwdWarps * 32, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    int64_t per_group =
        static_cast<int64_t>(sm_count(device)) * (per_sm > 0 ? per_sm : 1) / groups;
    if (per_group < 1) per_group = 1;
    const int64_t needed = ceil_div(rows, kGroupFwdWarps);
    if (per_group > needed) per_group = needed;
    k.fwd_grouped<<<static_cast<unsigned>(per_group * groups), kGroupFwdWarps * 32, smem, s>>>(
        left, right, weight, output, rows, L, mags, groups, per_group * kGroupFwdWarps, vec2);
    e = cudaGetLastError();
    return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "tp_forward launch");
  }
  const bool want_staged = strcmp(variant, "staged") == 0;
  const StagedPlan sp = want_staged ? plan_staged(device, rows, L, full, 2, 0) : StagedPlan{};
  if (sp.ok && al16) {
    if ((st = allow_smem(reinterpret_cast<const void*>(k.fwd_staged), sp.smem)) != ICTC_OK)
      return st;
    k.fwd_staged<<<static_cast<unsigned>(sp.grid), sp.warps * 32, sp.smem, s>>>(
        left, right, weight, output, rows, L, mags, sp.groups, sp.R, sp.stages);
  } else {
    const bool vec2 = (L.width % 2 == 0) && aligned(left, 8) && aligned(right, 8) &&
                      aligned(output, 8);
    DirectPlan g;
    st = plan_direct(reinterpret_cast<const void*>(k.fwd_direct), device, rows, channels, full,
                     &g);
    if (st != ICTC_OK) return st;
    k.fwd_direct<<<static_cast<unsigned>(g.blocks), kDirectThreads, 0, s>>>(
        left, right, weight, output, rows, L, mags, g.groups, g.nwarps, g.slots, vec2);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tp_forward launch");
  return ICTC_OK;
}

}  // namespace

extern "C" int32_t ictc_o2_tp_forward(const float* left, const float* right, const float* weight,
                                      float* output, int64_t rows, int32_t channels,
                                      int32_t m_max, int32_t parity, int32_t normalization,
                                      void* stream) {
  return tp_forward_impl(left, right, weight, output, rows, channels, m_max, parity,
                         normalization, ICTC_LAYOUT_CHANNEL_MAJOR, stream);
}

extern "C" int32_t ictc_o2_tp_forward_layout(const float* left, const float* right,
                                             const float* weight, float* output, int64_t rows,
                                             int32_t channels, int32_t m_max, int32_t parity,
                                             int32_t normalization, int32_t layout,
                                             void* stream) {
  return tp_forward_impl(left, right, weight, output, rows, channels, m_max, parity,
                         normalization, layout, stream);
}

extern "C" int32_t ictc_o2_tp_backward_workspace(int64_t rows, int32_t channels, int32_t m_max,
                                                 int32_t parity, int32_t device, size_t* bytes) {
  if (bytes == nullptr) return fail(ICTC_ERR_INVALID, "bytes is null");
  int st = validate(rows, channels, m_max, parity, ICTC_NORM_COMPONENT);
  if (st != ICTC_OK) return st;
  if (rows == 0) {
    *bytes = 0;
    return ICTC_OK;
  }
  int prev = 0;
  if ((st = current_device(&prev)) != ICTC_OK) return st;
  if (device != prev) {
    const cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  }
  const bool full = parity == ICTC_PARITY_FULL;
  // the larger of the two layouts' needs (their kernels' launch plans may differ)
  int64_t slots = 0;
  size_t chunk_bytes = 0;
  for (int cm = 0; cm < 2 && st == ICTC_OK; ++cm) {
    const TpLayout L = tp_layout(channels, m_max, full, cm);
    const Kernels& k = kKernels.k[cm][full ? 1 : 0][m_max];
    const int64_t s = backward_slots(device, k, rows, L, full, &st);
    if (s > slots) slots = s;
    const size_t c = weight_chunk_bytes(k, channels, full);
    if (c > chunk_bytes) chunk_bytes = c;
  }
  if (device != prev) cudaSetDevice(prev);
  if (st != ICTC_OK) return st;
  const int64_t numel = weight_numel(channels, m_max, full);
  *bytes = chunk_bytes + static_cast<size_t>(slots) * numel * sizeof(float);
  return ICTC_OK;
}

namespace {

int32_t tp_backward_impl(const float* left, const float* right, const float* weight,
                         const float* grad_output, float* grad_left, float* grad_right,
                         float* grad_weight, void* workspace, size_t workspace_bytes,
                         int64_t rows, int32_t channels, int32_t m_max, int32_t parity,
                         int32_t normalization, int32_t layout, void* stream) {
  int st = validate(rows, channels, m_max, parity, normalization);
  if (st != ICTC_OK) return st;
  if (layout != ICTC_LAYOUT_CHANNEL_MAJOR && layout != ICTC_LAYOUT_COMPONENT_MAJOR)
    return fail(ICTC_ERR_INVALID, "layout must be ICTC_LAYOUT_CHANNEL_MAJOR or _COMPONENT_MAJOR");
  if (!grad_weight) return fail(ICTC_ERR_INVALID, "grad_weight is null");
  const bool full = parity == ICTC_PARITY_FULL;
  const int64_t numel = weight_numel(channels, m_max, full);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    const int64_t blocks = ceil_div(numel, 256) < 1024 ? ceil_div(numel, 256) : 1024;
    zero_kernel<<<static_cast<unsigned>(blocks > 0 ? blocks : 1), 256, 0, s>>>(grad_weight, numel);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "zero launch");
  }
  if (!left || !right || !weight || !grad_output || !grad_left || !grad_right || !workspace)
    return fail(ICTC_ERR_INVALID, "null tensor pointer");
  if (!aligned(left, 4) || !aligned(right, 4) || !aligned(weight, 4) ||
      !aligned(grad_output, 4) || !aligned(grad_left, 4) || !aligned(grad_right, 4) ||
      !aligned(grad_weight, 4) || !aligned(workspace, 16))
    return fail(ICTC_ERR_INVALID, "tensor pointers must be 4-byte aligned (workspace 16)");
  const TpLayout L = tp_layout(channels, m_max, full, layout);
  const Kernels& k = kKernels.k[L.cm][full ? 1 : 0][m_max];
  int device = 0;
  if ((st = current_device(&device)) != ICTC_OK) return st;
  const size_t wbytes = weight_chunk_bytes(k, channels, full);
  const bool al16 = aligned16({left, right, grad_output, grad_left, grad_right});
  const char* bwd_variant = getenv("ICTC_TP_BACKWARD");
  const bool allow_tiled = bwd_variant == nullptr || strcmp(bwd_variant, "tiled") == 0;
  const TiledPlan tp = (al16 && allow_tiled) ? plan_tiled(device, rows, L, full, k.chunks)
                                             : TiledPlan{};
  RowTileMaps maps{};
  bool tiled = tp.ok;
  if (tiled) {
    const float* ops[3] = {left, right, grad_output};
    for (int t = 0; t < 3 && tiled; ++t)
      tiled = encode_row_tile_maps(ops[t], rows, channels, m_max, full, L.cm != 0, L.width,
                                   tp.Ct, &maps.m[2 * t]) == 0;
  }
  const StagedPlan sp = tiled ? StagedPlan{} : plan_staged_backward(device, k, rows, L, full);
  const bool staged = !tiled && sp.ok && al16;
  DirectPlan dp{};
  if (!staged && !tiled) {
    st = plan_direct(reinterpret_cast<const void*>(k.bwd_direct), device, rows, channels, full,
                     &dp);
    if (st != ICTC_OK) return st;
  }
  const int64_t slots = tiled ? tp.ctas * tp.R : (staged ? sp.grid * sp.R : dp.slots);
  const size_t need = wbytes + static_cast<size_t>(slots) * numel * sizeof(float);
  if (workspace_bytes < need)
    return fail(ICTC_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, need);
  float4* chunks = static_cast<float4*>(workspace);
  float* partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + wbytes);
  const Mags mags = tp_mags(normalization);
  const int groups = static_cast<int>(ceil_div(channels, full ? 16 : 32));
  k.prescale<<<dim3(static_cast<unsigned>(ceil_div(groups * 32, 256)),
                   static_cast<unsigned>(k.chunks)),
               256, 0, s>>>(weight, chunks, L,
                                                                               mags, groups);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prescale launch");
  if (tiled) {
    if ((st = allow_smem(reinterpret_cast<const void*>(k.bwd_tiled), tp.smem)) != ICTC_OK)
      return st;
    const TpLayout Lt = tp_layout(tp.Ct, m_max, full, layout);
    k.bwd_tiled<<<static_cast<unsigned>(tp.grid), kStagedWarps * 32, tp.smem, s>>>(
        maps, chunks, grad_left, grad_right, partial, numel, rows, L, Lt, mags, tp.gt, tp.R,
        tp.stages, tp.ntiles, tp.weights_in_smem ? 1 : 0);
  } else if (staged) {
    const BackwardStagedFn fn = sp.paired ? k.bwd_paired : k.bwd_staged;
    if ((st = allow_smem(reinterpret_cast<const void*>(fn), sp.smem)) != ICTC_OK) return st;
    fn<<<static_cast<unsigned>(sp.grid), sp.warps * 32, sp.smem, s>>>(
        left, right, chunks, grad_output, grad_left, grad_right, partial, numel, rows, L, mags,
        sp.groups, sp.R, sp.stages, sp.weights_in_smem ? 1 : 0);
  } else {
    const bool vec2 = (L.width % 2 == 0) && aligned(left, 8) && aligned(right, 8) &&
                      aligned(grad_output, 8) && aligned(grad_left, 8) && aligned(grad_right, 8);
    k.bwd_direct<<<static_cast<unsigned>(dp.blocks), kDirectThreads, 0, s>>>(
        left, right, chunks, grad_output, grad_left, grad_right, partial, numel, rows, L, mags,
        dp.groups, dp.nwarps, dp.slots, vec2);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tp_backward launch");
  reduce_slots_kernel<<<static_cast<unsigned>(ceil_div(numel, 32)), 256, 0, s>>>(
      partial, grad_weight, numel, slots);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "reduce launch");
  return ICTC_OK;
}

}  // namespace

extern "C" int32_t ictc_o2_tp_backward(const float* left, const float* right, const float* weight,
                                       const float* grad_output, float* grad_left,
                                       float* grad_right, float* grad_weight, void* workspace,
                                       size_t workspace_bytes, int64_t rows, int32_t channels,
                                       int32_t m_max, int32_t parity, int32_t normalization,
                                       void* stream) {
  return tp_backward_impl(left, right, weight, grad_output, grad_left, grad_right, grad_weight,
                          workspace, workspace_bytes, rows, channels, m_max, parity,
                          normalization, ICTC_LAYOUT_CHANNEL_MAJOR, stream);
}

extern "C" int32_t ictc_o2_tp_backward_layout(
    const float* left, const float* right, const float* weight, const float* grad_output,
    float* grad_left, float* grad_right, float* grad_weight, void* workspace,
    size_t workspace_bytes, int64_t rows, int32_t channels, int32_t m_max, int32_t parity,
    int32_t normalization, int32_t layout, void* stream) {
  return tp_backward_impl(left, right, weight, grad_output, grad_left, grad_right, grad_weight,
                          workspace, workspace_bytes, rows, channels, m_max, parity,
                          normalization, layout, stream);
}

// ------------------------------------------------------------ no-alloc backward
//
// Some callers cannot allocate device memory at the point where they need the
// backward pass: a host runtime whose allocator is owned by someone else (a
// framework pool that must not be bypassed, an embedded engine that reserved all
// device memory up front) or code running under a policy that forbids
// cudaMalloc/cudaFree on the hot path.  They get ictc_o2_tp_backward_noalloc: the
// same kernels and launch plan as ictc_o2_tp_backward, with the workspace taken
// from a fixed array in device global memory that the library owns.
//
// The array is kTpNoAllocScratchBytes (32 MiB) per GPU; every GPU on which the
// library's module is loaded holds it until the process exits.  Host code must
// not hand the array's name to a kernel (on the host the name is only a stand-in
// for the device symbol), so the first call on each device looks up the device
// address with cudaGetSymbolAddress while that device is current and caches it.
// That first call should therefore be made before any stream capture begins.
//
// Nothing in the array has to start at zero: the prescale kernel rewrites the
// weight chunks on every call, and every slot's partial weight-gradient row is
// written in full before the slot reduction reads it.  All calls on a device
// share the one array, so calls whose kernels overlap on the GPU (concurrent
// streams, or several host threads) race on it; the caller must order them.

namespace ictc {
namespace {

constexpr size_t kTpNoAllocScratchBytes = size_t(32) << 20;
constexpr int kTpNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_tp_noalloc_scratch[kTpNoAllocScratchBytes];

std::mutex g_tp_noalloc_mutex;
void* g_tp_noalloc_address[kTpNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once).
int tp_noalloc_scratch(int device, void** address) {
  if (device < 0 || device >= kTpNoAllocMaxDevices)
    return fail(ICTC_ERR_UNSUPPORTED, "device ordinal %d beyond the %d supported", device,
                kTpNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_tp_noalloc_mutex);
  if (g_tp_noalloc_address[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_tp_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (backward scratch)");
    g_tp_noalloc_address[device] = p;
  }
  *address = g_tp_noalloc_address[device];
  return ICTC_OK;
}

}  // namespace
}  // namespace ictc

extern "C" int32_t ictc_o2_tp_backward_noalloc(const float* left, const float* right,
                                               const float* weight, const float* grad_output,
                                               float* grad_left, float* grad_right,
                                               float* grad_weight, int64_t rows, int32_t channels,
                                               int32_t m_max, int32_t parity,
                                               int32_t normalization, void* stream) {
  int st = validate(rows, channels, m_max, parity, normalization);
  if (st != ICTC_OK) return st;
  if (rows == 0)  // writes a zero grad_weight; needs no workspace
    return ictc_o2_tp_backward(left, right, weight, grad_output, grad_left, grad_right,
                               grad_weight, nullptr, 0, rows, channels, m_max, parity,
                               normalization, stream);
  int device = 0;
  if ((st = current_device(&device)) != ICTC_OK) return st;
  size_t need = 0;
  if ((st = ictc_o2_tp_backward_workspace(rows, channels, m_max, parity, device, &need)) !=
      ICTC_OK)
    return st;
  if (need > kTpNoAllocScratchBytes)
    return fail(ICTC_ERR_WORKSPACE,
                "no-alloc backward: channels=%d m_max=%d needs %zu bytes of scratch, more than "
                "the fixed %zu; call ictc_o2_tp_backward with a caller workspace instead",
                channels, m_max, need, kTpNoAllocScratchBytes);
  void* scratch = nullptr;
  if ((st = tp_noalloc_scratch(device, &scratch)) != ICTC_OK) return st;
  return ictc_o2_tp_backward(left, right, weight, grad_output, grad_left, grad_right, grad_weight,
                             scratch, kTpNoAllocScratchBytes, rows, channels, m_max, parity,
                             normalization, stream);
}
