// Path table of the O(2) uvu product (host side), packed for the kernels.
//
// Reference: src/ictc_o2_hp/uvu_o2.py:27-156.  Entries are the copies of each
// block ([copy, channel, component] storage, uvu_o2.py:27-41).  Paths are every
// legal (first entry i, second entry j, output entry k), ordered by k, then i,
// then j (uvu_o2.py:122-137).  Coefficients are the normalised CG tensor with the
// reflection-twisted copy bases applied (J for copy 1, uvu_o2.py:44-47, 128-135),
// stored padded as c[k][a][b] (uvu_o2.py:134-135), divided by sqrt(V * count_k)
// under path normalization (uvu_o2.py:138-144).
#pragma once

#include <cmath>
#include <cstdint>
#include <vector>

#include "o2_paths.cuh"

namespace ictc {

constexpr int kUvuMaxEntries = 2 + 2 * 32;

struct UvuEntryH {
  int key;     // 0: 0e, -1: 0o, m >= 1: frequency m
  int copy;    // 0 or 1
  int offset;  // in the flat row
  int dim;     // 1 or 2
};

struct UvuPathH {
  int i, j, k;
  float c[8];  // c[kc * 4 + a * 2 + b]
};

struct UvuTableH {
  int U = 0, V = 0, width1 = 0, width2 = 0;
  std::vector<UvuEntryH> in1, in2;
  std::vector<UvuPathH> paths;
  std::vector<int> by_i, by_j;  // stable orders of the path indices
};

inline std::vector<UvuEntryH> uvu_entries(int channels, int order, bool full, int* width) {
  std::vector<UvuEntryH> out;
  int cursor = 0;
  out.push_back({0, 0, cursor, 1});
  cursor += channels;
  if (full) {
    out.push_back({-1, 0, cursor, 1});
    cursor += channels;
  }
  for (int m = 1; m <= order; ++m) {
    const int copies = full ? 2 : 1;
    for (int q = 0; q < copies; ++q) out.push_back({m, q, cursor + q * channels * 2, 2});
    cursor += copies * channels * 2;
  }
  *width = cursor;
  return out;
}

inline bool uvu_valid(int k1, int k2, int k3) {
  if (k1 <= 0 && k2 <= 0) return k3 == (((k1 == -1) != (k2 == -1)) ? -1 : 0);
  if (k1 <= 0) return k3 == k2;
  if (k2 <= 0) return k3 == k1;
  if (k1 == k2) return k3 == 0 || k3 == -1 || k3 == 2 * k1;
  return k3 == (k1 > k2 ? k1 - k2 : k2 - k1) || k3 == k1 + k2;
}

// Dense normalised CG tensor cg[a][b][kc] (o2_paths.cuh closed form).
inline void uvu_cg(int k1, int k2, int k3, bool component, double cg[2][2][2]) {
  for (int a = 0; a < 2; ++a)
    for (int b = 0; b < 2; ++b)
      for (int c = 0; c < 2; ++c) cg[a][b][c] = 0.0;
  ChanPath p{};
  fill_terms(p, k1, k2, k3);
  double norm2 = 0.0;
  for (int t = 0; t < p.nt; ++t) norm2 += 1.0;
  const int d3 = k3 > 0 ? 2 : 1;
  const double scale = (component ? std::sqrt(static_cast<double>(d3)) : 1.0) / std::sqrt(norm2);
  for (int t = 0; t < p.nt; ++t) cg[p.t[t].i][p.t[t].j][p.t[t].k] = p.t[t].s * scale;
}

inline UvuTableH build_uvu_table(int U, int V, int m1, bool full1, int m2, bool full2,
                                 bool component, bool path_normalized) {
  UvuTableH tab;
  tab.U = U;
  tab.V = V;
  tab.in1 = uvu_entries(U, m1, full1, &tab.width1);
  tab.in2 = uvu_entries(V, m2, full2, &tab.width2);
  const double J[2][2] = {{0.0, -1.0}, {1.0, 0.0}};
  auto basis = [&](const UvuEntryH& e, int r, int c) -> double {
    if (e.copy) return J[r][c];
    return r == c ? 1.0 : 0.0;
  };
  const int n1 = static_cast<int>(tab.in1.size());
  const int n2 = static_cast<int>(tab.in2.size());
  for (int k = 0; k < n1; ++k) {
    const UvuEntryH& out = tab.in1[k];
    const size_t start = tab.paths.size();
    for (int i = 0; i < n1; ++i) {
      const UvuEntryH& a = tab.in1[i];
      for (int j = 0; j < n2; ++j) {
        const UvuEntryH& b = tab.in2[j];
        if (!uvu_valid(a.key, b.key, out.key)) continue;
        double cg[2][2][2];
        uvu_cg(a.key, b.key, out.key, component, cg);
        UvuPathH p{};
        p.i = i;
        p.j = j;
        p.k = k;
        // c'[ai][bj][l] = sum cg[a][b][kc] B1[a][ai] B2[b][bj] Bout[kc][l], padded c[l][ai][bj]
        for (int l = 0; l < out.dim; ++l)
          for (int ai = 0; ai < a.dim; ++ai)
            for (int bj = 0; bj < b.dim; ++bj) {
              double s = 0.0;
              for (int aa = 0; aa < a.dim; ++aa)
                for (int bb = 0; bb < b.dim; ++bb)
                  for (int kc = 0; kc < out.dim; ++kc)
                    s += cg[aa][bb][kc] * basis(a, aa, ai) * basis(b, bb, bj) * basis(out, kc, l);
              p.c[l * 4 + ai * 2 + bj] = static_cast<float>(s);
            }
        tab.paths.push_back(p);
      }
    }
    const size_t count = tab.paths.size() - start;
    if (path_normalized && count) {
      const double scale = std::sqrt(static_cast<double>(V) * static_cast<double>(count));
      for (size_t q = start; q < tab.paths.size(); ++q)
        for (float& c : tab.paths[q].c) c = static_cast<float>(c / scale);
    }
  }
  const int np = static_cast<int>(tab.paths.size());
  for (int e = 0; e < n1; ++e)
    for (int p = 0; p < np; ++p)
      if (tab.paths[p].i == e) tab.by_i.push_back(p);
  for (int e = 0; e < n2; ++e)
    for (int p = 0; p < np; ++p)
      if (tab.paths[p].j == e) tab.by_j.push_back(p);
  return tab;
}

// Packed device table (int32 words; coefficients as float bits).  Every section
// starts on a 16-byte boundary (the kernels read paths as int4):
//   [0..15]   n1, n2, np, U, V, width1, width2, 0,
//             off_in1, off_in2, off_paths, off_coef, off_by_i, off_by_j, words, 0
//   in1       n1 x (offset, dim)
//   in2       n2 x (offset, dim)
//   paths     np x (i, j, k, 0)
//   coef      np x 8 floats
//   by_i, by_j  np each
struct UvuLayout {
  int n1, n2, np;
  int in1, in2, paths, coef, by_i, by_j, words;
};

constexpr int align4(int words) { return (words + 3) & ~3; }

inline UvuLayout uvu_layout(int n1, int n2, int np) {
  UvuLayout l;
  l.n1 = n1;
  l.n2 = n2;
  l.np = np;
  l.in1 = 16;
  l.in2 = align4(l.in1 + 2 * n1);
  l.paths = align4(l.in2 + 2 * n2);
  l.coef = align4(l.paths + 4 * np);
  l.by_i = align4(l.coef + 8 * np);
  l.by_j = align4(l.by_i + np);
  l.words = align4(l.by_j + np);
  return l;
}

}  // namespace ictc
