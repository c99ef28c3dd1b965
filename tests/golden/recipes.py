"""Seeded input recipes of the full-size fixtures.

``make_golden.py`` runs the reference on these inputs (in this container, where the
reference source exists) and stores its float64 results; the GPU tests rebuild the
same inputs on the GPU box from the same seeds and compare the kernels with the
stored values.  Inputs come from numpy's ``Generator`` (PCG64), whose streams are
the same on every machine, so nothing but the seeds needs to be stored.

Shapes follow the benchmark configs:
- config 4: UvuTensorProduct(128, 32, 3, full), inputs iid N(0, 1), weights
  N(0, 1) / sqrt(32), shared (131,072 rows) or per row (16,384 rows);
- config 5: RadialUvuTensorProduct over a V = 1 uvu (C = 64, m_max = 3, full, angular
  canonical m_max = 3), 1,048,576 edges over 65,536 nodes with uniform random
  endpoints and no self-loops, r ~ U(0.5, 5.0), Bessel(8) x cosine cutoff 5.0 -> MLP
  8 -> 64 -> 64 (SiLU) for the hidden features, angular = the unit-direction
  harmonics [1, cos t, sin t, ..., cos 3t, sin 3t] of t ~ U(0, 2 pi).
"""

from __future__ import annotations

import math

import numpy as np

# ------------------------------------------------------------------ config 4

CFG4 = dict(u=128, v=32, m_max=3, width1=1792, width2=448, weight_numel=606208)
CFG4_SHARED_ROWS = 131072
CFG4_SHARED_SEED = 4
CFG4_SHARED_KEEP = (0, 1, 2, 4095, 4096, 65535, 99991, 131071)

CFG4_PERROW_ROWS = 16384
CFG4_PERROW_SEED = 44
# rows whose inputs come from their own numpy stream (the rest of the per-row
# batch is filled on the GPU): the first and last rows, both sides of 4096-row
# boundaries and a few in between
CFG4_PERROW_KEEP = (0, 1, 4095, 4096, 7001, 12288, 16382, 16383)
# entries of a per-row weight gradient kept in the fixture: every 37th of 606,208
CFG4_PERROW_DW_COLUMNS = range(0, 606208, 37)


def cfg4_shared_inputs():
    """(x [N, 1792], y [N, 448], w [606208], g [N, 1792]) float32."""
    c = CFG4
    rng = np.random.default_rng(CFG4_SHARED_SEED)
    n = CFG4_SHARED_ROWS
    x = rng.standard_normal((n, c["width1"]), dtype=np.float32)
    y = rng.standard_normal((n, c["width2"]), dtype=np.float32)
    w = (rng.standard_normal(c["weight_numel"]) / math.sqrt(c["v"])).astype(np.float32)
    g = rng.standard_normal((n, c["width1"]), dtype=np.float32)
    return x, y, w, g


def cfg4_perrow_row(row: int):
    """One row of the per-row case: (x [1792], y [448], w [606208], g [1792])."""
    c = CFG4
    rng = np.random.default_rng((CFG4_PERROW_SEED, row))
    x = rng.standard_normal(c["width1"], dtype=np.float32)
    y = rng.standard_normal(c["width2"], dtype=np.float32)
    w = (rng.standard_normal(c["weight_numel"]) / math.sqrt(c["v"])).astype(np.float32)
    g = rng.standard_normal(c["width1"], dtype=np.float32)
    return x, y, w, g


# ------------------------------------------------------------------ config 5

CFG5 = dict(u=64, m_max=3, hidden=64, edges=1048576, nodes=65536, rc=5.0, basis=8,
            width1=896, width2=7, weight_numel=4736)
CFG5_SEED = 5
CFG5_KEEP = (0, 1, 2, 8191, 8192, 524287, 777777, 1048575)


def _silu(v):
    return v / (1.0 + np.exp(-v))


def cfg5_inputs(edges: int | None = None):
    """Config-5 edge inputs.  Returns a dict with node features ``nodes``
    [65536, 896], ``src`` / ``dst`` (int64), ``angular`` [E, 7], ``hidden`` [E, 64],
    the affine layer ``alpha`` [4736, 64] and ``bias`` [4736], and the cotangent
    ``g`` [E, 896]; float arrays are float32.  The hidden features are computed in
    float64 and rounded once."""
    c = CFG5
    e = c["edges"] if edges is None else edges
    rng = np.random.default_rng(CFG5_SEED)
    nodes = rng.standard_normal((c["nodes"], c["width1"]), dtype=np.float32)
    src = rng.integers(0, c["nodes"], e)
    dst = (src + rng.integers(1, c["nodes"], e)) % c["nodes"]   # no self-loops
    r = rng.uniform(0.5, 5.0, e)
    theta = rng.uniform(0.0, 2 * math.pi, e)
    w1 = rng.standard_normal((c["basis"], c["hidden"])) / math.sqrt(c["basis"])
    b1 = 0.1 * rng.standard_normal(c["hidden"])
    w2 = rng.standard_normal((c["hidden"], c["hidden"])) / math.sqrt(c["hidden"])
    b2 = 0.1 * rng.standard_normal(c["hidden"])
    alpha = (rng.standard_normal((c["weight_numel"], c["hidden"]))
             / math.sqrt(c["hidden"])).astype(np.float32)
    bias = (0.1 * rng.standard_normal(c["weight_numel"])).astype(np.float32)
    g = rng.standard_normal((e, c["width1"]), dtype=np.float32)
    n = np.arange(1, c["basis"] + 1, dtype=np.float64)
    rc = c["rc"]
    basis = math.sqrt(2 / rc) * np.sin(n * math.pi * r[:, None] / rc) / r[:, None]
    basis *= (0.5 * (np.cos(math.pi * r / rc) + 1))[:, None]
    hidden = _silu(_silu(basis @ w1 + b1) @ w2 + b2).astype(np.float32)
    angular = np.concatenate(
        [np.ones((e, 1))] + [np.stack([np.cos(m * theta), np.sin(m * theta)], -1)
                             for m in range(1, c["m_max"] + 1)], axis=-1).astype(np.float32)
    return dict(nodes=nodes, src=src, dst=dst, angular=angular, hidden=hidden, alpha=alpha,
                bias=bias, g=g)
