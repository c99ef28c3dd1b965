"""Host-side algebra: closed-form CG tables, path enumeration and the compiled
kernel tables agree with the oracle and with the reference's golden tables."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from ictc_o2_hp_b200 import _algebra as A
from ictc_o2_hp_b200 import _lib
from oracle import o2_oracle as O


def _key(text):
    tag, value = text.split(":")
    return (tag, int(value))


@pytest.mark.parametrize("normalization", ["component", "norm"])
def test_closed_form_cg_matches_reference_tables(normalization):
    data = load_golden("cg_tables")
    for name, raw in zip(data["names"], data["cg"]):
        k1, k2, k3 = (_key(t) for t in str(name).split("|"))
        d3 = A.key_dim(k3)
        norm = np.linalg.norm(raw)
        expected = raw * (math.sqrt(d3) / norm if normalization == "component" else 1 / norm)
        got = A.cg_tensor(k1, k2, k3, normalization)
        padded = np.zeros((2, 2, 2))
        padded[:got.shape[0], :got.shape[1], :got.shape[2]] = got
        assert np.abs(padded - expected).max() < 1e-12, name


@pytest.mark.parametrize("parity", ["canonical", "full"])
@pytest.mark.parametrize("m_max", range(0, 9))
def test_plan_matches_oracle_paths(parity, m_max):
    plan = A.TpPlan(3, m_max, parity)
    oracle = O.TpOracle(3, m_max, parity)
    assert plan.weight_numel == oracle.weight_numel
    assert plan.representation_dimension == oracle.width
    assert len(plan.paths) == len(oracle.paths)
    for p, q in zip(plan.paths, oracle.paths):
        assert (p.key1, p.key2, p.key3, p.weight_start, p.weight_stop) == q[:5]
        dense = A.cg_tensor(p.key1, p.key2, p.key3)
        assert np.abs(dense - q[6]).max() < 1e-12


@pytest.mark.parametrize("parity", ["canonical", "full"])
@pytest.mark.parametrize("m_max", range(0, 9))
def test_compiled_table_matches_plan(parity, m_max):
    plan = A.TpPlan(5, m_max, parity)
    compiled = _lib.tp_path_table(m_max, parity)
    expected = plan.kernel_table()
    assert len(compiled) == len(expected)
    for got, want in zip(compiled, expected):
        assert got[:6] == want[:6]
        assert sorted(got[6]) == sorted(want[6])
    for channels in (1, 17, 128):
        assert _lib.tp_weight_numel(channels, m_max, parity) == A.TpPlan(
            channels, m_max, parity).weight_numel


def test_known_answer_path_counts():
    """P, W and weight counts quoted for the benchmark configs."""
    p1 = A.TpPlan(32, 2, "canonical")
    assert (len(p1.paths), p1.representation_dimension, p1.weight_numel) == (10, 160, 320)
    p2 = A.TpPlan(128, 6, "full")
    assert (len(p2.paths), p2.representation_dimension, p2.weight_numel) == (85, 3328, 19712)
    terms = sum(len(p.terms) * (p.weight_stop - p.weight_start) for p in p2.paths)
    assert terms == 61952


@pytest.mark.parametrize("name", [n for n in golden_names("tp_") if "cfg" not in n])
def test_seeded_init_matches_reference(name):
    from ictc_o2_hp_b200 import TensorProduct
    case = load_golden(name)
    torch.manual_seed(int(case["seed"]))
    tp = TensorProduct(int(case["channels"]), int(case["m_max"]), parity=str(case["parity"]),
                       normalization=str(case["normalization"]))
    assert np.array_equal(tp.weight.detach().numpy(), case["weight"])
    assert [str(p) for p in tp.paths] == [str(p) for p in case["paths"]]


def test_module_attributes_and_state_dict():
    from ictc_o2_hp_b200 import TensorProduct
    tp = TensorProduct(32, 2, parity="canonical")
    keys = list(tp.state_dict().keys())
    assert keys == ["weight"] + [f"cg_{i}" for i in range(10)] + ["odd_to_even", "even_to_odd"]
    assert tp.state_dict()["cg_0"].dtype == torch.float64
    assert tp.parameter_count == 320
    assert tp.representation_spec()[1] == {"labels": "1", "frequency": 1, "irrep_dimension": 2,
                                           "multiplicity": 32, "parity_copies": 1}
    full = TensorProduct(4, 2)
    assert full.representation_spec()[2]["labels"] == "1e+1o"
    # load_state_dict round trip
    other = TensorProduct(32, 2, parity="canonical")
    other.load_state_dict(tp.state_dict())
    assert torch.equal(other.weight, tp.weight)


def test_errors_without_cuda():
    from ictc_o2_hp_b200 import TensorProduct
    tp = TensorProduct(4, 1)
    x = torch.randn(2, tp.representation_dimension)
    with pytest.raises(TypeError, match="CUDA float32"):
        tp(x, x)
    with pytest.raises(ValueError, match="configured width"):
        tp(x[:, :-1], x[:, :-1])
    with pytest.raises(ValueError):
        TensorProduct(0, 1)
    with pytest.raises(ValueError):
        TensorProduct(4, -1)
    with pytest.raises(ValueError):
        TensorProduct(4, 1, parity="odd")
