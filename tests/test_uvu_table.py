"""The library's uvu path table (ictc_o2_uvu_table) agrees with the Python plan and
with the oracle (paths, entries, coefficients, orders), and the module mirrors the
reference's attributes and validation."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ictc_o2_hp_b200 import UvuTensorProduct, _lib
from oracle import o2_oracle as O

CONFIGS = [
    # channels, channels_in2, m_max, parity, m_max_in2, parity_in2, normalization, path_norm
    (128, 32, 3, "full", 3, "full", "component", "none"),
    (64, 1, 3, "full", 3, "canonical", "component", "none"),
    (5, 2, 2, "canonical", 2, "canonical", "norm", "path"),
    (4, 3, 3, "full", 2, "canonical", "component", "element"),
    (7, 5, 6, "full", 4, "full", "norm", "none"),
    (3, 2, 0, "full", 1, "canonical", "component", "none"),
]


def unpack(table):
    n1, n2, np_, U, V, w1, w2 = (int(v) for v in table[:7])
    o_in1, o_in2, o_paths, o_coef, o_bi, o_bj, words = (int(v) for v in table[8:15])
    assert words == len(table)
    for off in (o_in1, o_in2, o_paths, o_coef, o_bi, o_bj):
        assert off % 4 == 0  # 16-byte aligned sections
    return dict(U=U, V=V, w1=w1, w2=w2,
                in1=table[o_in1:o_in1 + 2 * n1].reshape(n1, 2),
                in2=table[o_in2:o_in2 + 2 * n2].reshape(n2, 2),
                paths=table[o_paths:o_paths + 4 * np_].reshape(np_, 4)[:, :3],
                coef=table[o_coef:o_coef + 8 * np_].view(np.float32).reshape(np_, 2, 2, 2),
                by_i=table[o_bi:o_bi + np_], by_j=table[o_bj:o_bj + np_])


@pytest.mark.parametrize("cfg", CONFIGS)
def test_table_matches_plan_and_oracle(cfg):
    U, V, m1, p1, m2, p2, norm, pnorm = cfg
    tp = UvuTensorProduct(U, V, m1, parity=p1, m_max_in2=m2, parity_in2=p2,
                          normalization=norm, path_normalization=pnorm)
    t = unpack(tp._table.numpy())
    oracle = O.UvuOracle(U, V, m1, p1, p2, m2, norm, pnorm)
    assert (t["U"], t["V"], t["w1"], t["w2"]) == (U, V, tp.input1_dimension, tp.input2_dimension)
    assert np.array_equal(t["paths"], np.array(tp.paths).reshape(-1, 3))
    assert np.array_equal(t["paths"], np.array(oracle.paths).reshape(-1, 3))
    assert np.abs(t["coef"] - oracle.coefficients).max() < 1e-6
    assert np.abs(tp._coefficient_values - oracle.coefficients).max() < 1e-12
    assert [tuple(e) for e in t["in1"]] == [(e.offset, e.dim) for e in tp.entries_in1]
    assert [tuple(e) for e in t["in2"]] == [(e.offset, e.dim) for e in tp.entries_in2]
    paths = np.array(tp.paths).reshape(-1, 3)
    assert list(t["by_i"]) == sorted(range(len(paths)), key=lambda p: paths[p][0])
    assert list(t["by_j"]) == sorted(range(len(paths)), key=lambda p: paths[p][1])


def test_known_answer_counts():
    """Path and weight counts of the benchmark configs 4 and 5."""
    tp = UvuTensorProduct(128, 32, 3)
    assert (len(tp.paths), tp.weight_numel, tp.input1_dimension, tp.input2_dimension) == \
        (148, 606208, 1792, 448)
    radial = UvuTensorProduct(64, 1, 3, parity_in2="canonical", shared_weights=False)
    assert (len(radial.paths), radial.weight_numel, radial.input1_dimension,
            radial.input2_dimension) == (74, 4736, 896, 7)


def test_module_api_and_validation():
    torch.manual_seed(0)
    tp = UvuTensorProduct(6, 2, 2)
    assert tp.weight.shape == (tp.weight_numel,) and tp.parameter_count == tp.weight_numel
    assert list(tp.state_dict().keys()) == ["weight"]
    view = tp.weight_view_for_path(3)
    assert view.shape == (6, 2)
    ext = UvuTensorProduct(6, 1, 2, shared_weights=False)
    assert ext.parameter_count == 0 and ext.weight.numel() == 0
    with pytest.raises(ValueError):
        UvuTensorProduct(6, 1, 2, shared_weights=False, internal_weights=True)
    with pytest.raises(ValueError):
        UvuTensorProduct(0, 1, 2)
    with pytest.raises(ValueError):
        UvuTensorProduct(2, 1, 2, normalization="bad")
    x = torch.randn(3, tp.input1_dimension)
    y = torch.randn(3, tp.input2_dimension)
    with pytest.raises(TypeError, match="CUDA float32"):
        tp(x, y)
    with pytest.raises(ValueError, match="input1_dimension"):
        tp(x[:, :-1], y)
    with pytest.raises(ValueError, match="external weights"):
        ext(x, torch.randn(3, ext.input2_dimension))
