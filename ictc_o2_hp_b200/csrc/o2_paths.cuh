// Compile-time O(2) path tables for the fused TensorProduct kernels.
//
// The reference builds its Clebsch-Gordan ("Cartesian/Fischer") coefficients
// numerically from Gaussian-Gram harmonic projections (o2_math.py:86-346) and
// expands them into sparse (i, j, k, coef) terms (fast_o2.py:16-36).  Every
// such tensor is a signed complex product with one magnitude per path:
//
//   * a frequency-m vector (a0, a1) is the amplitude A = s_m (a0 + i a1) of the
//     harmonic Re(conj(A) (x + i y)^m), with s_m = +1 for m mod 4 in {1, 2} and
//     -1 for m mod 4 in {0, 3} (the reference's sign fixing, o2_math.py:130-133);
//   * F(m1) x F(m2) -> F(m1 + m2) is A1 A2, -> F(|m1 - m2|) is A1 conj(A2)
//     (m1 > m2) or conj(A1) A2 (m2 > m1), each times s_m1 s_m2 s_m3;
//   * F(m) x F(m) -> 0e is Re(conj(A1) A2), -> 0o is the antisymmetric form
//     (o2_math.py:282-293); scalar x frequency uses I (0e) or J^T (0o)
//     (o2_math.py:310-333).
//
// The signs live here as compile-time tables; the per-path magnitude (1, 1/sqrt2
// or 1/2, set by the normalization, native_o2.py:118-123) is a runtime scalar
// folded into the weight.  The path order and packed weight offsets follow
// native_o2.py:101-117 / fast_o2.py:157-167: for key1 in keys, key2 in keys, for
// key3 in the valid outputs (o2_math.py:348-372) that are active.
//
// Per channel c the computation is closed over the "slot" vector
//   slot 0 = 0e[c], slot 1 = 0o[c], slots 2m, 2m+1 = frequency m (one copy).
// Full parity has two copies per frequency.  Cyclic routing (native_o2.py:128-129)
// makes copy q of a frequency output read copy q of frequency inputs and the
// (copy-free) scalars, while scalar outputs read copy 0 only.  So a full-parity
// channel splits into two "parity worlds" q = 0, 1 that run the same frequency-
// output paths on their own copy; scalar-output paths exist only in world 0.
#pragma once

#include <cstdint>
#include <type_traits>
#include <utility>

namespace ictc {

constexpr int kMaxOrder = 8;        // largest m_max with a compiled fast kernel
constexpr int kMaxPaths = 160;      // >= path count of full parity at kMaxOrder

// Path classes; the magnitude of every term of a path depends only on its class.
enum PathClass : int { kSS = 0, kSF = 1, kFFS = 2, kFFF = 3 };

struct Term {
  int i, j, k, s;  // first-input component, second-input component, output component, sign
};

struct ChanPath {
  int in1, in2, out;  // slot index of component 0 of each operand
  int cls;            // PathClass
  int unit;           // packed weight offset in units of `channels`
  int copied;         // 1: frequency output in full parity (weight index adds copy * channels)
  int nt;             // number of sparse terms (1, 2 or 4)
  Term t[4];
};

struct PathTable {
  int n = 0;          // number of block paths
  int units = 0;      // weight.numel() / channels
  ChanPath p[kMaxPaths] = {};
};

// Basis sign of frequency m (see header comment).
constexpr int basis_sign(int m) { return (m % 4 == 1 || m % 4 == 2) ? 1 : -1; }

// Key encoding: 0 -> 0e, -1 -> 0o, m >= 1 -> frequency m.
constexpr int slot_of(int key) { return key == 0 ? 0 : (key == -1 ? 1 : 2 * key); }

constexpr void set_terms(ChanPath& c, int n, const int (*t)[4]) {
  c.nt = n;
  for (int q = 0; q < n; ++q) c.t[q] = Term{t[q][0], t[q][1], t[q][2], t[q][3]};
}

// Fill the sparse signed terms of key1 x key2 -> key3 (unit magnitude).
constexpr void fill_terms(ChanPath& c, int k1, int k2, int k3) {
  const bool s1 = k1 <= 0, s2 = k2 <= 0, s3 = k3 <= 0;
  if (s1 && s2) {
    const int t[1][4] = {{0, 0, 0, 1}};
    c.cls = kSS;
    set_terms(c, 1, t);
  } else if (s1 && !s2) {  // scalar x frequency -> frequency
    c.cls = kSF;
    if (k1 == 0) {
      const int t[2][4] = {{0, 0, 0, 1}, {0, 1, 1, 1}};
      set_terms(c, 2, t);
    } else {
      const int t[2][4] = {{0, 0, 1, 1}, {0, 1, 0, -1}};
      set_terms(c, 2, t);
    }
  } else if (!s1 && s2) {  // frequency x scalar -> frequency
    c.cls = kSF;
    if (k2 == 0) {
      const int t[2][4] = {{0, 0, 0, 1}, {1, 0, 1, 1}};
      set_terms(c, 2, t);
    } else {
      const int t[2][4] = {{0, 0, 1, 1}, {1, 0, 0, -1}};
      set_terms(c, 2, t);
    }
  } else if (s3) {  // frequency x frequency -> scalar (m1 == m2)
    c.cls = kFFS;
    if (k3 == 0) {
      const int t[2][4] = {{0, 0, 0, 1}, {1, 1, 0, 1}};
      set_terms(c, 2, t);
    } else {
      const int t[2][4] = {{0, 1, 0, 1}, {1, 0, 0, -1}};
      set_terms(c, 2, t);
    }
  } else {  // frequency x frequency -> frequency
    c.cls = kFFF;
    const int g = basis_sign(k1) * basis_sign(k2) * basis_sign(k3);
    if (k3 == k1 + k2) {  // A1 A2: (a0 b0 - a1 b1, a0 b1 + a1 b0)
      const int t[4][4] = {{0, 0, 0, g}, {1, 1, 0, -g}, {0, 1, 1, g}, {1, 0, 1, g}};
      set_terms(c, 4, t);
    } else if (k1 > k2) {  // A1 conj(A2): (a0 b0 + a1 b1, a1 b0 - a0 b1)
      const int t[4][4] = {{0, 0, 0, g}, {1, 1, 0, g}, {1, 0, 1, g}, {0, 1, 1, -g}};
      set_terms(c, 4, t);
    } else {  // conj(A1) A2: (a0 b0 + a1 b1, a0 b1 - a1 b0)
      const int t[4][4] = {{0, 0, 0, g}, {1, 1, 0, g}, {0, 1, 1, g}, {1, 0, 1, -g}};
      set_terms(c, 4, t);
    }
  }
}

constexpr PathTable build_table(int m_max, bool full) {
  PathTable tab{};
  int keys[2 + kMaxOrder] = {};
  int nk = 0;
  keys[nk++] = 0;
  if (full) keys[nk++] = -1;
  for (int m = 1; m <= m_max; ++m) keys[nk++] = m;
  int unit = 0;
  for (int a = 0; a < nk; ++a) {
    for (int b = 0; b < nk; ++b) {
      const int k1 = keys[a], k2 = keys[b];
      int outs[3] = {};
      int no = 0;
      if (k1 <= 0 && k2 <= 0) {
        outs[no++] = ((k1 == -1) != (k2 == -1)) ? -1 : 0;
      } else if (k1 <= 0) {
        outs[no++] = k2;
      } else if (k2 <= 0) {
        outs[no++] = k1;
      } else if (k1 == k2) {
        outs[no++] = 0;
        outs[no++] = -1;
        outs[no++] = 2 * k1;
      } else {
        outs[no++] = k1 > k2 ? k1 - k2 : k2 - k1;
        outs[no++] = k1 + k2;
      }
      for (int o = 0; o < no; ++o) {
        const int k3 = outs[o];
        if (k3 == -1 && !full) continue;  // 0o inactive in canonical parity
        if (k3 > m_max) continue;         // frequency truncation
        ChanPath& c = tab.p[tab.n++];
        c.in1 = slot_of(k1);
        c.in2 = slot_of(k2);
        c.out = slot_of(k3);
        c.unit = unit;
        c.copied = (full && k3 > 0) ? 1 : 0;
        fill_terms(c, k1, k2, k3);
        unit += c.copied ? 2 : 1;
      }
    }
  }
  tab.units = unit;
  return tab;
}

// A permutation of the paths of a table.
struct PathOrder {
  int idx[kMaxPaths] = {};
};

// Kernel execution order: paths with a frequency output (run by both parity
// worlds) first, then the scalar-output paths (world 0 only, one divergent
// region in full parity); inside each part, grouped by first-input slot, which
// shortens register live ranges in the adjoint.
constexpr PathOrder by_first_input(const PathTable& t) {
  PathOrder o{};
  int n = 0;
  for (int part = 0; part < 2; ++part)
    for (int slot = 0; slot <= 2 * kMaxOrder + 1; ++slot)
      for (int p = 0; p < t.n; ++p)
        if (t.p[p].in1 == slot && (t.p[p].out >= 2) == (part == 0)) o.idx[n++] = p;
  return o;
}

// Number of leading entries of by_first_input() with a frequency output.
constexpr int frequency_output_paths(const PathTable& t) {
  int n = 0;
  for (int p = 0; p < t.n; ++p) n += t.p[p].out >= 2 ? 1 : 0;
  return n;
}

template <int M, bool FULL>
struct Paths {
  static constexpr PathTable table = build_table(M, FULL);
  static constexpr int n = table.n;
  static constexpr int slots = 2 * M + 2;
  static constexpr PathOrder vjp = by_first_input(table);
  static constexpr int nfreq = frequency_output_paths(table);
  static constexpr int chunks = (n + 3) / 4;  // float4 chunks of per-thread weights
};

// Compile-time loop: f(std::integral_constant<int, I>) for I in [0, N).
template <int N, typename F, int... I>
__host__ __device__ __forceinline__ void static_for_impl(F&& f, std::integer_sequence<int, I...>) {
  (f(std::integral_constant<int, I>{}), ...);
}
template <int N, typename F>
__host__ __device__ __forceinline__ void static_for(F&& f) {
  static_for_impl<N>(static_cast<F&&>(f), std::make_integer_sequence<int, N>{});
}

}  // namespace ictc
