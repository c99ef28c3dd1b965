"""O(2) representation blocks, path enumeration and closed-form CG coefficients.

This is the host-side description of the algebra the compiled kernels implement
(csrc/o2_paths.cuh).  It reproduces, in closed form, the reference's numerically
built Cartesian Clebsch-Gordan tensors (reference: src/ictc_o2_hp/o2_math.py:86-346,
normalised in native_o2.py:118-123):

* a frequency-m vector (a0, a1) is the amplitude ``A = s_m (a0 + i a1)`` of the
  harmonic ``Re(conj(A) (x + i y)^m)`` with ``s_m = +1`` for ``m % 4 in (1, 2)`` and
  ``-1`` otherwise (the sign convention fixed in o2_math.py:76-84, 130-133);
* ``F(m1) x F(m2) -> F(m1 + m2)`` is ``A1 A2``; ``-> F(|m1 - m2|)`` is ``A1 conj(A2)``
  (m1 > m2) or ``conj(A1) A2`` (m2 > m1), each times ``s_m1 s_m2 s_m3``;
* ``F(m) x F(m) -> 0e`` is ``Re(conj(A1) A2)``, ``-> 0o`` is ``a0 b1 - a1 b0``
  (o2_math.py:282-293); scalar x frequency uses the identity (0e) or ``J^T`` (0o)
  (o2_math.py:310-333); scalar x scalar is 1.

Every term of a path then has one magnitude: 1, 1/sqrt(2) or 1/2 depending on the
path class and the normalization.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Iterable

import numpy as np

O2Key = tuple  # ("scalar", +1 | -1) or ("freq", m >= 1)

SCALAR_EVEN: O2Key = ("scalar", 1)
SCALAR_ODD: O2Key = ("scalar", -1)

# Path classes, shared with the kernels (o2_paths.cuh PathClass).
CLASS_SS, CLASS_SF, CLASS_FFS, CLASS_FFF = 0, 1, 2, 3

_R = 1.0 / math.sqrt(2.0)
# Magnitude of every term per class: component normalization scales each CG
# tensor to norm sqrt(dim_out), "norm" to norm 1 (native_o2.py:118-123).
MAGNITUDES = {
    "component": (1.0, 1.0, _R, _R),
    "norm": (1.0, _R, _R, 0.5),
}


@dataclass(frozen=True)
class RepresentationBlock:
    """One irrep block of a flat row (reference: native_o2.py:26-33)."""

    token: str
    key: O2Key
    frequency: int
    irrep_dimension: int
    multiplicity: int
    parity_copies: int


def full_parity_blocks(max_frequency: int, channels: int) -> tuple[RepresentationBlock, ...]:
    """0e, 0o and two reflection copies per positive frequency (native_o2.py:35-49)."""
    if max_frequency < 0:
        raise ValueError("max_frequency must be non-negative")
    if channels <= 0:
        raise ValueError("channels must be positive")
    blocks = [RepresentationBlock("0e", SCALAR_EVEN, 0, 1, channels, 1),
              RepresentationBlock("0o", SCALAR_ODD, 0, 1, channels, 1)]
    blocks += [RepresentationBlock(str(m), ("freq", m), m, 2, 2 * channels, 2)
               for m in range(1, max_frequency + 1)]
    return tuple(blocks)


def canonical_blocks(max_frequency: int, channels: int) -> tuple[RepresentationBlock, ...]:
    """0e and one copy per positive frequency (native_o2.py:52-61)."""
    if max_frequency < 0 or channels <= 0:
        raise ValueError("invalid frequency or channels")
    return (RepresentationBlock("0e", SCALAR_EVEN, 0, 1, channels, 1),
            *(RepresentationBlock(f"{m}", ("freq", m), m, 2, channels, 1)
              for m in range(1, max_frequency + 1)))


def normalize_key(key) -> O2Key:
    """Accepts ("scalar", +-1), ("freq", m) or the tokens "0e", "0o", "m"."""
    if isinstance(key, tuple):
        tag, value = str(key[0]).strip().lower(), int(key[1])
        if tag == "scalar" and value in (-1, 1):
            return ("scalar", value)
        if tag == "freq" and value >= 1:
            return ("freq", value)
        raise ValueError(f"Invalid O(2) key {key!r}")
    token = str(key).strip().lower()
    if token == "0e":
        return SCALAR_EVEN
    if token == "0o":
        return SCALAR_ODD
    if token.isdigit() and int(token) >= 1:
        return ("freq", int(token))
    raise ValueError(f"Invalid O(2) irrep token {key!r}")


def key_dim(key: O2Key) -> int:
    return 1 if key[0] == "scalar" else 2


def valid_output_keys(key1, key2) -> list[O2Key]:
    """Irreps in key1 (x) key2, in the reference's order (o2_math.py:348-372)."""
    k1, k2 = normalize_key(key1), normalize_key(key2)
    if k1[0] == "scalar" and k2[0] == "scalar":
        return [("scalar", k1[1] * k2[1])]
    if k1[0] == "scalar":
        return [k2]
    if k2[0] == "scalar":
        return [k1]
    m1, m2 = k1[1], k2[1]
    if m1 == m2:
        return [SCALAR_EVEN, SCALAR_ODD, ("freq", 2 * m1)]
    return [("freq", abs(m1 - m2)), ("freq", m1 + m2)]


def basis_sign(m: int) -> int:
    return 1 if m % 4 in (1, 2) else -1


def path_class(key1: O2Key, key2: O2Key, key3: O2Key) -> int:
    s1, s2, s3 = (k[0] == "scalar" for k in (key1, key2, key3))
    if s1 and s2:
        return CLASS_SS
    if s1 or s2:
        return CLASS_SF
    return CLASS_FFS if s3 else CLASS_FFF


def signed_terms(key1, key2, key3) -> tuple[tuple[int, int, int, int], ...]:
    """Sparse unit-magnitude terms (i, j, k, sign) of key1 x key2 -> key3, or () if
    the coupling vanishes."""
    k1, k2, k3 = normalize_key(key1), normalize_key(key2), normalize_key(key3)
    if k3 not in valid_output_keys(k1, k2):
        return ()
    if k1[0] == "scalar" and k2[0] == "scalar":
        return ((0, 0, 0, 1),)
    if k1[0] == "scalar":
        return ((0, 0, 0, 1), (0, 1, 1, 1)) if k1[1] == 1 else ((0, 0, 1, 1), (0, 1, 0, -1))
    if k2[0] == "scalar":
        return ((0, 0, 0, 1), (1, 0, 1, 1)) if k2[1] == 1 else ((0, 0, 1, 1), (1, 0, 0, -1))
    if k3 == SCALAR_EVEN:
        return ((0, 0, 0, 1), (1, 1, 0, 1))
    if k3 == SCALAR_ODD:
        return ((0, 1, 0, 1), (1, 0, 0, -1))
    m1, m2, m3 = k1[1], k2[1], k3[1]
    g = basis_sign(m1) * basis_sign(m2) * basis_sign(m3)
    if m3 == m1 + m2:
        return ((0, 0, 0, g), (1, 1, 0, -g), (0, 1, 1, g), (1, 0, 1, g))
    if m1 > m2:
        return ((0, 0, 0, g), (1, 1, 0, g), (1, 0, 1, g), (0, 1, 1, -g))
    return ((0, 0, 0, g), (1, 1, 0, g), (0, 1, 1, g), (1, 0, 1, -g))


def cg_tensor(key1, key2, key3, normalization: str = "component") -> np.ndarray:
    """Dense normalised CG tensor [d1, d2, d3] in float64 (zeros when it vanishes)."""
    k1, k2, k3 = normalize_key(key1), normalize_key(key2), normalize_key(key3)
    out = np.zeros((key_dim(k1), key_dim(k2), key_dim(k3)), dtype=np.float64)
    terms = signed_terms(k1, k2, k3)
    if not terms:
        return out
    mag = MAGNITUDES[normalization][path_class(k1, k2, k3)]
    for i, j, k, s in terms:
        out[i, j, k] = s * mag
    return out


@dataclass(frozen=True)
class TpPath:
    """A block path of TensorProduct with its packed weight slice."""

    key1: O2Key
    key2: O2Key
    key3: O2Key
    weight_start: int
    weight_stop: int
    cls: int
    terms: tuple


class TpPlan:
    """Blocks, keys, paths and packed-weight layout of TensorProduct(channels, m_max,
    parity, normalization), in the reference's order (native_o2.py:101-117,
    fast_o2.py:152-167)."""

    def __init__(self, channels: int, m_max: int, parity: str = "full",
                 normalization: str = "component"):
        if parity not in ("canonical", "full"):
            raise ValueError(parity)
        if normalization not in MAGNITUDES:
            raise ValueError(normalization)
        self.channels, self.m_max = int(channels), int(m_max)
        self.parity, self.normalization = parity, normalization
        self.full = parity == "full"
        self.blocks = (full_parity_blocks if self.full else canonical_blocks)(
            self.m_max, self.channels)
        self.keys = tuple(b.key for b in self.blocks)
        self.block_by_key = {b.key: b for b in self.blocks}
        active = set(self.keys)
        paths, cursor = [], 0
        for k1 in self.keys:
            for k2 in self.keys:
                for k3 in valid_output_keys(k1, k2):
                    if k3 not in active:
                        continue
                    mul = self.block_by_key[k3].multiplicity
                    paths.append(TpPath(k1, k2, k3, cursor, cursor + mul,
                                        path_class(k1, k2, k3), signed_terms(k1, k2, k3)))
                    cursor += mul
        self.paths = tuple(paths)
        self.weight_numel = cursor
        self.representation_dimension = sum(b.multiplicity * b.irrep_dimension
                                            for b in self.blocks)

    def key_offsets(self) -> dict:
        offsets, cursor = {}, 0
        for b in self.blocks:
            offsets[b.key] = cursor
            cursor += b.multiplicity * b.irrep_dimension
        return offsets

    def kernel_table(self) -> list[tuple]:
        """The table the compiled library should hold (ictc_o2_tp_path_table): per
        path (in1 slot, in2 slot, out slot, class, unit offset, copied, terms)."""
        def slot(key):
            return 0 if key == SCALAR_EVEN else (1 if key == SCALAR_ODD else 2 * key[1])
        rows = []
        for p in self.paths:
            copied = int(self.full and p.key3[0] == "freq")
            rows.append((slot(p.key1), slot(p.key2), slot(p.key3), p.cls,
                         p.weight_start // self.channels, copied, tuple(p.terms)))
        return rows


def iter_entries(blocks: Iterable[RepresentationBlock], channels: int):
    """Yields (key, copy, offset, dim) for each copy of each block, offsets in the
    flat row (reference: uvu_o2.py:27-41)."""
    cursor = 0
    for block in blocks:
        for copy in range(block.parity_copies):
            yield block.key, copy, cursor + copy * channels * block.irrep_dimension, \
                block.irrep_dimension
        cursor += block.multiplicity * block.irrep_dimension


# --------------------------------------------------------------------------- uvu


@dataclass(frozen=True)
class UvuEntry:
    """One representation copy (reference: uvu_o2.py:14-18)."""

    key: O2Key
    copy: int
    offset: int
    dim: int


def uvu_representation(channels: int, order: int, parity: str):
    """(blocks, entries, width) of one uvu operand (uvu_o2.py:27-41)."""
    if parity not in ("canonical", "full"):
        raise ValueError("parity must be canonical or full")
    blocks = (canonical_blocks if parity == "canonical" else full_parity_blocks)(order, channels)
    entries, cursor = [], 0
    for block in blocks:
        for copy in range(block.parity_copies):
            entries.append(UvuEntry(block.key, copy,
                                    cursor + copy * channels * block.irrep_dimension,
                                    block.irrep_dimension))
        cursor += block.multiplicity * block.irrep_dimension
    return blocks, tuple(entries), cursor


_J = np.array([[0.0, -1.0], [1.0, 0.0]])


def _copy_basis(entry: UvuEntry) -> np.ndarray:
    return _J if entry.copy else np.eye(entry.dim)


def uvu_paths(entries_in1, entries_in2, normalization: str, path_normalization: str,
              channels_in2: int):
    """Paths (i, j, k) ordered by output entry, first entry, second entry and their
    padded coefficients c[p, k, a, b] in float64 (uvu_o2.py:121-145)."""
    paths, coefficients = [], []
    for k, out in enumerate(entries_in1):
        start = len(paths)
        for i, first in enumerate(entries_in1):
            for j, second in enumerate(entries_in2):
                if out.key not in valid_output_keys(first.key, second.key):
                    continue
                cg = cg_tensor(first.key, second.key, out.key, normalization)
                cg = np.einsum("abk,ai,bj,lk->ijl", cg, _copy_basis(first),
                               _copy_basis(second), _copy_basis(out).T)
                padded = np.zeros((2, 2, 2))
                padded[:out.dim, :first.dim, :second.dim] = np.transpose(cg, (2, 0, 1))
                paths.append((i, j, k))
                coefficients.append(padded)
        count = len(paths) - start
        if path_normalization != "none":
            scale = math.sqrt(channels_in2 * count)
            for p in range(start, len(paths)):
                coefficients[p] = coefficients[p] / scale
    coef = np.stack(coefficients) if coefficients else np.zeros((0, 2, 2, 2))
    return tuple(paths), coef
