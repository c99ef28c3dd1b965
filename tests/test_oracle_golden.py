"""Pins the CPU oracle to the reference: every golden fixture (made by running the
reference, tests/golden/make_golden.py) must be reproduced by oracle/o2_oracle.py."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_names, load_golden
from oracle import o2_oracle as O

TOL_F64 = 1e-11


def _key(text):
    tag, value = text.split(":")
    return (tag, int(value))


def test_cg_tables_match_reference():
    data = load_golden("cg_tables")
    assert len(data["names"]) > 100
    for name, ref in zip(data["names"], data["cg"]):
        k1, k2, k3 = (_key(t) for t in str(name).split("|"))
        cg = O.cg_tensor(k1, k2, k3)
        padded = np.zeros((2, 2, 2))
        padded[:cg.shape[0], :cg.shape[1], :cg.shape[2]] = cg
        assert np.abs(padded - ref).max() < 1e-12, name


def replay_tp_inputs(case):
    """Regenerates the benchmark-recipe inputs: torch.manual_seed(seed), the module's
    weight init (one randn(out_mul) per path, native_o2.py:110-117), then x, y."""
    import torch
    oracle = O.TpOracle(int(case["channels"]), int(case["m_max"]), str(case["parity"]),
                        str(case["normalization"]))
    torch.manual_seed(int(case["seed"]))
    weights = [torch.randn(e - s) * 0.02 for (_, _, _, s, e, _, _) in oracle.paths]
    rows = int(case["torch_rows"])
    x = torch.randn(rows, oracle.width)
    y = torch.randn(rows, oracle.width)
    return oracle, torch.cat(weights).numpy(), x.numpy(), y.numpy()


@pytest.mark.parametrize("name", [n for n in golden_names("tp_") if "cfg" not in n])
def test_tp_oracle_matches_reference(name):
    case = load_golden(name)
    oracle = O.TpOracle(int(case["channels"]), int(case["m_max"]), str(case["parity"]),
                        str(case["normalization"]))
    assert [str(p) for p in case["paths"]] == [str((p[0], p[1], p[2])) for p in oracle.paths]
    x, y = case["x"].astype(np.float64), case["y"].astype(np.float64)
    w = case["weight"].astype(np.float64)
    g = case["g"].astype(np.float64)
    out, dx, dy, dw = oracle.vjp(x, y, w, g)
    for key, value in (("out", out), ("dx", dx), ("dy", dy), ("dw", dw)):
        assert O.max_error(value, case[f"{key}_f64"]) < TOL_F64, key
    if "out_f32" in case:  # the reference's FP32 path agrees with f64 within 1e-5
        for key, value in (("out", out), ("dx", dx), ("dy", dy), ("dw", dw)):
            assert O.max_error(value, case[f"{key}_f32"]) < 1e-5, key


def test_tp_config1_recipe_replay():
    """Config 1 (TP(32,2,canonical), seed 0, N=4096, ones cotangent) in full."""
    case = load_golden("tp_c32_m2_canonical_cfg1")
    oracle, w, x, y = replay_tp_inputs(case)
    assert np.array_equal(w.astype(np.float32), case["weight"])
    g = np.ones_like(x, dtype=np.float64)
    out, dx, dy, dw = oracle.vjp(x.astype(np.float64), y.astype(np.float64),
                                 w.astype(np.float64), g)
    rows = case["keep_rows"]
    for key, value in (("out", out), ("dx", dx), ("dy", dy)):
        assert O.max_error(value[rows], case[f"{key}_f64_rows"]) < TOL_F64, key
        assert O.max_error(value.sum(axis=0), case[f"{key}_f64_sum"]) < 1e-9, key
    assert O.max_error(dw, case["dw_f64"]) < 1e-9


def test_tp_config2_recipe_rows():
    """Config 2 (TP(128,6,full), seed 0, N=65536): the kept rows of out, dx, dy."""
    case = load_golden("tp_c128_m6_full_cfg2")
    oracle, w, x, y = replay_tp_inputs(case)
    assert np.array_equal(w.astype(np.float32), case["weight"])
    rows = case["keep_rows"]
    xs, ys = x[rows].astype(np.float64), y[rows].astype(np.float64)
    out, dx, dy, _ = oracle.vjp(xs, ys, w.astype(np.float64), np.ones_like(xs))
    for key, value in (("out", out), ("dx", dx), ("dy", dy)):
        assert O.max_error(value, case[f"{key}_f64_rows"]) < TOL_F64, key


@pytest.mark.parametrize("name", golden_names("uvu_"))
def test_uvu_oracle_matches_reference(name):
    case = load_golden(name)
    oracle = O.UvuOracle(int(case["u"]), int(case["v"]), int(case["m_max"]),
                         str(case["parity"]), str(case["parity_in2"]),
                         int(case["m_max_in2"]), str(case["normalization"]),
                         str(case["path_normalization"]))
    assert np.array_equal(np.array(oracle.paths), case["paths"])
    assert np.abs(oracle.coefficients - case["coefficients"]).max() < 1e-12
    shared = bool(case["shared"])
    args = [case[k].astype(np.float64) for k in ("x", "y", "w", "g")]
    out, dx, dy, dw = oracle.vjp(*args, shared=shared)
    for key, value in (("out", out), ("dx", dx), ("dy", dy), ("dw", dw)):
        assert O.max_error(value, case[f"{key}_f64"]) < TOL_F64, key


@pytest.mark.parametrize("name", golden_names("radial_"))
def test_radial_oracle_matches_reference(name):
    case = load_golden(name)
    uvu = O.UvuOracle(int(case["u"]), 1, int(case["m_max"]), "full", "canonical")
    radial = O.RadialOracle(uvu)
    bias = case["b"].astype(np.float64) if bool(case["bias"]) else None
    f = {k: case[k].astype(np.float64) for k in ("x", "y", "h", "alpha", "g")}
    out, dx, dy, dh, da, db = radial.vjp(f["x"], f["y"], f["h"], f["alpha"], f["g"], bias)
    for key, value in (("out", out), ("dx", dx), ("dy", dy), ("dh", dh), ("da", da)):
        assert O.max_error(value, case[f"{key}_f64"]) < TOL_F64, key
    if bias is not None:
        assert O.max_error(db, case["db_f64"]) < TOL_F64


def test_max_error_metric():
    assert O.max_error([1.0, 2.0], [1.0, 2.0]) == 0.0
    assert abs(O.max_error([1.0, 2.0], [1.0, 2.2]) - 0.2 / 2.2) < 1e-12
    assert O.max_error([0.0], [1e-9]) == pytest.approx(1e-2)
