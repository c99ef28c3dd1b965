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
// A warp keeps the same channel group for its whole life (the grid holds a
// multiple of `groups` warps), so its path weights stay in registers in the
// forward pass and its weight-gradient accumulators stay in registers in the
// backward pass.  The weight gradient is reduced deterministically: each warp
// slot writes one partial row, then a second kernel sums the slots in a fixed
// order (reference: two-stage FP32 reduction, triton_o2.py:744-780, 948-959).
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "o2_paths.cuh"

namespace ictc {

namespace {

constexpr int kThreads = 128;  // 4 warps per CTA
#ifndef ICTC_FENCE_EVERY
#define ICTC_FENCE_EVERY 8
#endif
constexpr int kFenceEvery = ICTC_FENCE_EVERY;

__device__ __forceinline__ float2 ld2(const float* p, bool vec2) {
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

// Slot vector of channel c in world q, in the canonical basis: the odd copy
// (r0, r1) is read as (-r1, r0) (reference fast_o2.py:61-66).
template <int M, bool FULL>
__device__ __forceinline__ void load_slots(const float* __restrict__ row, const TpLayout& L,
                                           int c, int q, bool vec2, float (&v)[2 * M + 2]) {
  v[0] = __ldg(row + c);
  v[1] = FULL ? __ldg(row + L.C + c) : 0.0f;
#pragma unroll
  for (int m = 1; m <= M; ++m) {
    const float2 r = ld2(row + L.fbase + (m - 1) * L.fstride + 2 * (q * L.C + c), vec2);
    v[2 * m] = q ? -r.y : r.x;
    v[2 * m + 1] = q ? r.x : r.y;
  }
}

// Writes the frequency slots of world q; the odd copy (v0, v1) is stored as
// (v1, -v0) (reference fast_o2.py:68-73).  Scalars are written by world 0.
template <int M, bool FULL>
__device__ __forceinline__ void store_slots(float* __restrict__ row, const TpLayout& L, int c,
                                            int q, bool vec2, const float (&v)[2 * M + 2]) {
  if (q == 0) {
    row[c] = v[0];
    if (FULL) row[L.C + c] = v[1];
  }
#pragma unroll
  for (int m = 1; m <= M; ++m) {
    float* p = row + L.fbase + (m - 1) * L.fstride + 2 * (q * L.C + c);
    st2(p, q ? v[2 * m + 1] : v[2 * m], q ? -v[2 * m] : v[2 * m + 1], vec2);
  }
}

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
  constexpr ChanPath cp = Paths<M, FULL>::table.p[I];
  float s[2];
  static_for<cp.nt>([&](auto T) {
    constexpr Term t = Paths<M, FULL>::table.p[I].t[T];
    mac<first_term<M, FULL, I, T, 0>(), t.s>(s[t.k], a[Paths<M, FULL>::table.p[I].in1 + t.i],
                                              b[Paths<M, FULL>::table.p[I].in2 + t.j]);
  });
  o[cp.out] = fmaf(w, s[0], o[cp.out]);
  if constexpr (slot_dim(cp.out) == 2) o[cp.out + 1] = fmaf(w, s[1], o[cp.out + 1]);
}

// First-order adjoint of path I for one row: dx, dy and the weight-gradient
// accumulator.  Three algebraically equal factorizations; the cheapest for the
// path's shape is chosen at compile time:
//   form 0:  s_k = sum a b,  acc += g.s,  dx_i += (w g_k) b_j,  dy_j += (w g_k) a_i
//   form 1/2: t_i = sum b_j g_k,  u_j = sum a_i g_k,  dx += w t,  dy += w u,
//             acc += a.t (form 1) or b.u (form 2)
template <int M, bool FULL, int I>
__device__ __forceinline__ void path_vjp(const float* a, const float* b, const float* g,
                                         float* dx, float* dy, float& acc, float w) {
  constexpr ChanPath cp = Paths<M, FULL>::table.p[I];
  constexpr int d1 = slot_dim(cp.in1), d2 = slot_dim(cp.in2), d3 = slot_dim(cp.out);
  constexpr int cost0 = 2 * d3 + 3 * cp.nt;
  constexpr int cost1 = 2 * cp.nt + 2 * d1 + d2;
  constexpr int cost2 = 2 * cp.nt + d1 + 2 * d2;
  if constexpr (cost0 <= cost1 && cost0 <= cost2) {
    float s[2];
    static_for<cp.nt>([&](auto T) {
      constexpr Term t = Paths<M, FULL>::table.p[I].t[T];
      mac<first_term<M, FULL, I, T, 0>(), t.s>(s[t.k], a[Paths<M, FULL>::table.p[I].in1 + t.i],
                                                b[Paths<M, FULL>::table.p[I].in2 + t.j]);
    });
    float wg[2];
    acc = fmaf(g[cp.out], s[0], acc);
    wg[0] = w * g[cp.out];
    if constexpr (d3 == 2) {
      acc = fmaf(g[cp.out + 1], s[1], acc);
      wg[1] = w * g[cp.out + 1];
    }
    static_for<cp.nt>([&](auto T) {
      constexpr Term t = Paths<M, FULL>::table.p[I].t[T];
      constexpr int i1 = Paths<M, FULL>::table.p[I].in1 + t.i;
      constexpr int i2 = Paths<M, FULL>::table.p[I].in2 + t.j;
      mac<false, t.s>(dx[i1], wg[t.k], b[i2]);
      mac<false, t.s>(dy[i2], wg[t.k], a[i1]);
    });
  } else {
    float tv[2], uv[2];
    static_for<cp.nt>([&](auto T) {
      constexpr Term t = Paths<M, FULL>::table.p[I].t[T];
      constexpr int i1 = Paths<M, FULL>::table.p[I].in1 + t.i;
      constexpr int i2 = Paths<M, FULL>::table.p[I].in2 + t.j;
      constexpr int i3 = Paths<M, FULL>::table.p[I].out + t.k;
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

template <int M, bool FULL>
__global__ void __launch_bounds__(kThreads)
    tp_forward_kernel(const float* __restrict__ x, const float* __restrict__ y,
                      const float* __restrict__ w, float* __restrict__ out, int64_t rows,
                      TpLayout L, Mags mags, int groups, int64_t nwarps, int64_t slots,
                      bool vec2) {
  using P = Paths<M, FULL>;
  constexpr int S = 2 * M + 2;
  constexpr int CPW = FULL ? 16 : 32;
  const int lane = threadIdx.x & 31;
  const int q = FULL ? (lane >> 4) : 0;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (gw >= nwarps) return;
  const int c_raw = static_cast<int>(gw % groups) * CPW + (FULL ? (lane & 15) : lane);
  const bool active = c_raw < L.C;
  const int c = active ? c_raw : 0;

  // Path weights of this channel and world, with the path magnitude folded in.
  float wr[P::n];
  static_for<P::n>([&](auto I) {
    constexpr ChanPath cp = P::table.p[I];
    const bool used = active && (!FULL || cp.copied || q == 0);
    wr[I] = used ? __ldg(w + weight_index<M, FULL, I>(L.C, c, q)) * mags.m[cp.cls] : 0.0f;
  });

  for (int64_t row = gw / groups; row < rows; row += slots) {
    float a[S], b[S], o[S];
    load_slots<M, FULL>(x + row * L.width, L, c, q, vec2, a);
    load_slots<M, FULL>(y + row * L.width, L, c, q, vec2, b);
#pragma unroll
    for (int s = 0; s < S; ++s) o[s] = 0.0f;
    static_for<P::n>([&](auto I) {
      if (FULL && !P::table.p[I].copied && q != 0) return;  // scalar outputs: world 0 only
      path_forward<M, FULL, I>(a, b, o, wr[I]);
    });
    if (active) store_slots<M, FULL>(out + row * L.width, L, c, q, vec2, o);
  }
}

template <int M, bool FULL>
__global__ void __launch_bounds__(kThreads)
    tp_backward_kernel(const float* __restrict__ x, const float* __restrict__ y,
                       const float* __restrict__ ws, const float* __restrict__ go,
                       float* __restrict__ gx, float* __restrict__ gy,
                       float* __restrict__ partial, int64_t numel, int64_t rows, TpLayout L,
                       Mags mags, int groups, int64_t nwarps, int64_t slots, bool vec2) {
  using P = Paths<M, FULL>;
  constexpr int S = 2 * M + 2;
  constexpr int CPW = FULL ? 16 : 32;
  const int lane = threadIdx.x & 31;
  const int q = FULL ? (lane >> 4) : 0;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (gw >= nwarps) return;  // whole warps only: nwarps counts warps
  const int c_raw = static_cast<int>(gw % groups) * CPW + (FULL ? (lane & 15) : lane);
  const bool active = c_raw < L.C;
  const int c = active ? c_raw : 0;
  const int64_t slot = gw / groups;

  float acc[P::n];
#pragma unroll
  for (int i = 0; i < P::n; ++i) acc[i] = 0.0f;

  for (int64_t row = slot; row < rows; row += slots) {
    float a[S], b[S], g[S], dx[S], dy[S];
    load_slots<M, FULL>(x + row * L.width, L, c, q, vec2, a);
    load_slots<M, FULL>(y + row * L.width, L, c, q, vec2, b);
    // The output twist (v0, v1) -> (v1, -v0) has the adjoint g -> (-g1, g0),
    // which is the same map as the input read.
    load_slots<M, FULL>(go + row * L.width, L, c, q, vec2, g);
#pragma unroll
    for (int s = 0; s < S; ++s) {
      dx[s] = 0.0f;
      dy[s] = 0.0f;
    }
    static_for<P::n>([&](auto I) {
      if (FULL && !P::table.p[I].copied && q != 0) return;  // scalar outputs: world 0 only
      const float wv = ld_stream(ws + weight_index<M, FULL, I>(L.C, c, q));
      path_vjp<M, FULL, I>(a, b, g, dx, dy, acc[I], wv);
      // Scheduling fence: keeps the weight loads of later paths from being
      // issued early, which would raise register pressure past the budget.
      if constexpr (I % kFenceEvery == kFenceEvery - 1) asm volatile("" ::: "memory");
    });
    if (FULL) {
      // World 1 reaches the scalars through scalar x frequency paths.
      dx[0] += __shfl_xor_sync(0xffffffffu, dx[0], 16);
      dx[1] += __shfl_xor_sync(0xffffffffu, dx[1], 16);
      dy[0] += __shfl_xor_sync(0xffffffffu, dy[0], 16);
      dy[1] += __shfl_xor_sync(0xffffffffu, dy[1], 16);
    }
    if (active) {
      store_slots<M, FULL>(gx + row * L.width, L, c, q, vec2, dx);
      store_slots<M, FULL>(gy + row * L.width, L, c, q, vec2, dy);
    }
  }

  if (active) {
    float* dst = partial + slot * numel;
    static_for<P::n>([&](auto I) {
      constexpr ChanPath cp = P::table.p[I];
      if (FULL && !cp.copied && q != 0) return;
      dst[weight_index<M, FULL, I>(L.C, c, q)] = acc[I] * mags.m[cp.cls];
    });
  }
}

// Class of each weight unit (a unit is `channels` consecutive weights).
struct UnitClasses {
  unsigned char cls[2 * kMaxPaths];
};

UnitClasses unit_classes(int m_max, bool full) {
  const PathTable t = build_table(m_max, full);
  UnitClasses u{};
  for (int p = 0; p < t.n; ++p) {
    u.cls[t.p[p].unit] = static_cast<unsigned char>(t.p[p].cls);
    if (t.p[p].copied) u.cls[t.p[p].unit + 1] = static_cast<unsigned char>(t.p[p].cls);
  }
  return u;
}

// ws[i] = w[i] * magnitude of its path, so the row loop needs no extra multiply.
__global__ void prescale_kernel(const float* __restrict__ w, float* __restrict__ ws, int64_t numel,
                                int C, UnitClasses uc, Mags mags) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < numel;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    ws[i] = w[i] * mags.m[uc.cls[i / C]];
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

struct Launch {
  int groups;
  int64_t slots;
  int64_t nwarps;
  int64_t blocks;
};

using ForwardFn = void (*)(const float*, const float*, const float*, float*, int64_t, TpLayout,
                           Mags, int, int64_t, int64_t, bool);
using BackwardFn = void (*)(const float*, const float*, const float*, const float*, float*,
                            float*, float*, int64_t, int64_t, TpLayout, Mags, int, int64_t,
                            int64_t, bool);

// ICTC_ONLY_ORDER=m builds one order only (quick register/spill checks).
#ifdef ICTC_ONLY_ORDER
constexpr bool compiled_order(int m) { return m == ICTC_ONLY_ORDER; }
#else
constexpr bool compiled_order(int) { return true; }
#endif

template <int M, bool FULL>
constexpr ForwardFn forward_ptr() {
  if constexpr (compiled_order(M)) return &tp_forward_kernel<M, FULL>;
  else return nullptr;
}
template <int M, bool FULL>
constexpr BackwardFn backward_ptr() {
  if constexpr (compiled_order(M)) return &tp_backward_kernel<M, FULL>;
  else return nullptr;
}

template <int... Ms>
constexpr auto make_forward_table(std::integer_sequence<int, Ms...>) {
  struct T { ForwardFn f[2][sizeof...(Ms)]; };
  return T{{{forward_ptr<Ms, false>()...}, {forward_ptr<Ms, true>()...}}};
}
template <int... Ms>
constexpr auto make_backward_table(std::integer_sequence<int, Ms...>) {
  struct T { BackwardFn f[2][sizeof...(Ms)]; };
  return T{{{backward_ptr<Ms, false>()...}, {backward_ptr<Ms, true>()...}}};
}

const auto kForward = make_forward_table(std::make_integer_sequence<int, kMaxOrder + 1>{});
const auto kBackward = make_backward_table(std::make_integer_sequence<int, kMaxOrder + 1>{});

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

// Workspace: [magnitude-scaled weights, padded to 256 B][slots x numel partials].
size_t scaled_weight_floats(int64_t numel) { return static_cast<size_t>(ceil_div(numel, 64) * 64); }
size_t backward_workspace_bytes(int64_t slots, int64_t numel) {
  return (scaled_weight_floats(numel) + static_cast<size_t>(slots) * static_cast<size_t>(numel)) *
         sizeof(float);
}

// Grid shape: a multiple of `groups` warps so that every warp keeps one channel
// group; `slots` warps share each group and split the rows round-robin.
int plan(const void* kernel, int64_t rows, int C, bool full, Launch* out) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  const int cpw = full ? 16 : 32;
  out->groups = static_cast<int>(ceil_div(C, cpw));
  const int64_t resident = static_cast<int64_t>(sm_count(device)) * (per_sm > 0 ? per_sm : 1) *
                           (kThreads / 32);
  int64_t slots = resident / out->groups;
  if (slots < 1) slots = 1;
  if (slots > rows) slots = rows > 0 ? rows : 1;
  out->slots = slots;
  out->nwarps = slots * out->groups;
  out->blocks = ceil_div(out->nwarps * 32, kThreads);
  return ICTC_OK;
}

}  // namespace

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

extern "C" int32_t ictc_o2_tp_forward(const float* left, const float* right, const float* weight,
                                      float* output, int64_t rows, int32_t channels,
                                      int32_t m_max, int32_t parity, int32_t normalization,
                                      void* stream) {
  int st = validate(rows, channels, m_max, parity, normalization);
  if (st != ICTC_OK) return st;
  if (rows == 0) return ICTC_OK;
  if (!left || !right || !weight || !output)
    return fail(ICTC_ERR_INVALID, "null tensor pointer");
  if (!aligned(left, 4) || !aligned(right, 4) || !aligned(weight, 4) || !aligned(output, 4))
    return fail(ICTC_ERR_INVALID, "tensor pointers must be 4-byte aligned");
  const bool full = parity == ICTC_PARITY_FULL;
  const TpLayout L = tp_layout(channels, m_max, full);
  const bool vec2 = (L.width % 2 == 0) && aligned(left, 8) && aligned(right, 8) &&
                    aligned(output, 8);
  ForwardFn fn = kForward.f[full ? 1 : 0][m_max];
  Launch g;
  st = plan(reinterpret_cast<const void*>(fn), rows, channels, full, &g);
  if (st != ICTC_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  fn<<<static_cast<unsigned>(g.blocks), kThreads, 0, s>>>(left, right, weight, output, rows, L,
                                                           tp_mags(normalization), g.groups,
                                                           g.nwarps, g.slots, vec2);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tp_forward launch");
  return ICTC_OK;
}

extern "C" int32_t ictc_o2_tp_backward_workspace(int64_t rows, int32_t channels, int32_t m_max,
                                                 int32_t parity, int32_t device, size_t* bytes) {
  if (bytes == nullptr) return fail(ICTC_ERR_INVALID, "bytes is null");
  int st = validate(rows, channels, m_max, parity, ICTC_NORM_COMPONENT);
  if (st != ICTC_OK) return st;
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (device != prev) {
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  }
  const bool full = parity == ICTC_PARITY_FULL;
  Launch g;
  st = plan(reinterpret_cast<const void*>(kBackward.f[full ? 1 : 0][m_max]), rows, channels,
            full, &g);
  if (device != prev) cudaSetDevice(prev);
  if (st != ICTC_OK) return st;
  *bytes = rows == 0 ? 0 : backward_workspace_bytes(g.slots, weight_numel(channels, m_max, full));
  return ICTC_OK;
}

extern "C" int32_t ictc_o2_tp_backward(const float* left, const float* right, const float* weight,
                                       const float* grad_output, float* grad_left,
                                       float* grad_right, float* grad_weight, void* workspace,
                                       size_t workspace_bytes, int64_t rows, int32_t channels,
                                       int32_t m_max, int32_t parity, int32_t normalization,
                                       void* stream) {
  int st = validate(rows, channels, m_max, parity, normalization);
  if (st != ICTC_OK) return st;
  if (!grad_weight) return fail(ICTC_ERR_INVALID, "grad_weight is null");
  const bool full = parity == ICTC_PARITY_FULL;
  const int64_t numel = weight_numel(channels, m_max, full);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    zero_kernel<<<static_cast<unsigned>(ceil_div(numel, 256) < 1024 ? ceil_div(numel, 256) : 1024),
                  256, 0, s>>>(grad_weight, numel);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ICTC_OK : cuda_fail(e, "zero launch");
  }
  if (!left || !right || !weight || !grad_output || !grad_left || !grad_right || !workspace)
    return fail(ICTC_ERR_INVALID, "null tensor pointer");
  if (!aligned(left, 4) || !aligned(right, 4) || !aligned(weight, 4) ||
      !aligned(grad_output, 4) || !aligned(grad_left, 4) || !aligned(grad_right, 4) ||
      !aligned(grad_weight, 4) || !aligned(workspace, 4))
    return fail(ICTC_ERR_INVALID, "tensor pointers must be 4-byte aligned");
  const TpLayout L = tp_layout(channels, m_max, full);
  const bool vec2 = (L.width % 2 == 0) && aligned(left, 8) && aligned(right, 8) &&
                    aligned(grad_output, 8) && aligned(grad_left, 8) && aligned(grad_right, 8);
  BackwardFn fn = kBackward.f[full ? 1 : 0][m_max];
  Launch g;
  st = plan(reinterpret_cast<const void*>(fn), rows, channels, full, &g);
  if (st != ICTC_OK) return st;
  const size_t need = backward_workspace_bytes(g.slots, numel);
  if (workspace_bytes < need)
    return fail(ICTC_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, need);
  float* scaled = static_cast<float*>(workspace);
  float* partial = scaled + scaled_weight_floats(numel);
  const Mags mags = tp_mags(normalization);
  prescale_kernel<<<static_cast<unsigned>(ceil_div(numel, 256) < 1024 ? ceil_div(numel, 256) : 1024),
                    256, 0, s>>>(weight, scaled, numel, channels, unit_classes(m_max, full), mags);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prescale launch");
  fn<<<static_cast<unsigned>(g.blocks), kThreads, 0, s>>>(
      left, right, scaled, grad_output, grad_left, grad_right, partial, numel, rows, L,
      mags, g.groups, g.nwarps, g.slots, vec2);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tp_backward launch");
  reduce_slots_kernel<<<static_cast<unsigned>(ceil_div(numel, 32)), 256, 0, s>>>(
      partial, grad_weight, numel, g.slots);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "reduce launch");
  return ICTC_OK;
}
