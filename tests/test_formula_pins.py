"""The differentiable PyTorch formulas of the three products (``ops.torch_tp_flat``,
``ops.torch_uvu_flat`` and the radial composition over it) are pinned to values the
reference itself produced (tests/golden/make_golden.py): first-order fixtures, and the
reference autograd's second derivatives (create_graph) of TensorProduct, uvu with
shared and per-row weights and the radial product.  These formulas are the float64
arbiters of the GPU second-derivative tests, so pinning them here means those tests
compare the kernels with reference-held values, not with this package's own algebra.
CPU only, float64; gate: normalised max error <= 1e-9 (the reference and the formula
differ only by float64 summation order)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import o2_oracle as O

TOL = 1e-9


def _t(a, grad=False):
    return torch.from_numpy(np.asarray(a)).double().requires_grad_(grad)


def _tp_formula(channels, m_max, parity, normalization):
    from ictc_o2_hp_b200.ops import tp_plan, torch_tp_flat
    plan = tp_plan(int(channels), int(m_max), str(parity), str(normalization))
    return lambda x, y, w: torch_tp_flat(x, y, w, plan)


def _uvu_formula(u, v, m_max, parity="full", parity_in2=None, m_max_in2=None,
                 normalization="component", path_normalization="none", shared=True):
    from ictc_o2_hp_b200 import UvuTensorProduct
    from ictc_o2_hp_b200.ops import torch_uvu_flat
    tp = UvuTensorProduct(int(u), int(v), int(m_max), parity=str(parity),
                          parity_in2=None if parity_in2 is None else str(parity_in2),
                          m_max_in2=None if m_max_in2 is None else int(m_max_in2),
                          normalization=str(normalization),
                          path_normalization=str(path_normalization), shared_weights=shared,
                          internal_weights=False)
    coef = torch.from_numpy(tp._coefficient_values).double()
    return lambda x, y, w: torch_uvu_flat(x, y, w, tp.entries_in1, tp.entries_in2, tp.paths,
                                          coef, int(u), int(v), shared)


def _radial_formula(u, m_max):
    inner = _uvu_formula(u, 1, m_max, parity="full", parity_in2="canonical", shared=False)

    def composed(x, y, h, a, b=None):
        w = h @ a.t()
        return inner(x, y, w if b is None else w + b)
    return composed


def _check(pairs):
    for name, got, want in pairs:
        err = O.max_error(got.detach().numpy(), want)
        assert err <= TOL, f"{name}: {err:.3e}"


@pytest.mark.parametrize("name", [n for n in golden_names("tp_") if "cfg" not in n])
def test_tp_formula_first_order(name):
    c = load_golden(name)
    f = _tp_formula(c["channels"], c["m_max"], c["parity"], c["normalization"])
    x, y, w = _t(c["x"], True), _t(c["y"], True), _t(c["weight"], True)
    out = f(x, y, w)
    grads = torch.autograd.grad(out, (x, y, w), _t(c["g"]))
    _check(zip(("out", "dx", "dy", "dw"), (out, *grads),
               (c[f"{k}_f64"] for k in ("out", "dx", "dy", "dw"))))


@pytest.mark.parametrize("name", golden_names("uvu_u"))
def test_uvu_formula_first_order(name):
    c = load_golden(name)
    shared = bool(c["shared"])
    f = _uvu_formula(c["u"], c["v"], c["m_max"], c["parity"], c["parity_in2"], c["m_max_in2"],
                     c["normalization"], c["path_normalization"], shared)
    x, y, w = _t(c["x"], True), _t(c["y"], True), _t(c["w"], True)
    out = f(x, y, w)
    grads = torch.autograd.grad(out, (x, y, w), _t(c["g"]))
    _check(zip(("out", "dx", "dy", "dw"), (out, *grads),
               (c[f"{k}_f64"] for k in ("out", "dx", "dy", "dw"))))


@pytest.mark.parametrize("name", [n for n in golden_names("radial_") if "cfg" not in n])
def test_radial_formula_first_order(name):
    c = load_golden(name)
    bias = bool(c["bias"])
    f = _radial_formula(c["u"], c["m_max"])
    ops = [_t(c[k], True) for k in ("x", "y", "h", "alpha")] + ([_t(c["b"], True)] if bias else [])
    out = f(*ops)
    grads = torch.autograd.grad(out, ops, _t(c["g"]))
    keys = ["out", "dx", "dy", "dh", "da"] + (["db"] if bias else [])
    _check(zip(keys, (out, *grads), (c[f"{k}_f64"] for k in keys)))


def _second(fn, operands, g, cotangents):
    first = torch.autograd.grad(fn(*operands), operands, g, create_graph=True)
    total = sum((f * h).sum() for f, h in zip(first, cotangents))
    return torch.autograd.grad(total, (*operands, g))


@pytest.mark.parametrize("name", golden_names("second_tp_"))
def test_tp_formula_second_order(name):
    c = load_golden(name)
    f = _tp_formula(c["channels"], c["m_max"], c["parity"], c["normalization"])
    ops = [_t(c[k], True) for k in ("x", "y", "w")]
    got = _second(f, ops, _t(c["g"], True), [_t(c[k]) for k in ("hx", "hy", "hw")])
    keys = ("sx", "sy", "sw", "sg")
    _check(zip(keys, got, (c[f"{k}_f64"] for k in keys)))


@pytest.mark.parametrize("name", golden_names("second_uvu_"))
def test_uvu_formula_second_order(name):
    c = load_golden(name)
    f = _uvu_formula(c["u"], c["v"], c["m_max"], shared=bool(c["shared"]))
    ops = [_t(c[k], True) for k in ("x", "y", "w")]
    got = _second(f, ops, _t(c["g"], True), [_t(c[k]) for k in ("hx", "hy", "hw")])
    keys = ("sx", "sy", "sw", "sg")
    _check(zip(keys, got, (c[f"{k}_f64"] for k in keys)))


@pytest.mark.parametrize("name", golden_names("second_radial_"))
def test_radial_formula_second_order(name):
    c = load_golden(name)
    bias = bool(c["bias"])
    f = _radial_formula(c["u"], c["m_max"])
    names = ["x", "y", "h", "alpha"] + (["b"] if bias else [])
    ops = [_t(c[k], True) for k in names]
    hs = [_t(c[k]) for k in ("hx", "hy", "hh", "ha")] + ([_t(c["hb"])] if bias else [])
    got = _second(f, ops, _t(c["g"], True), hs)
    keys = ["sx", "sy", "sh", "sa"] + (["sb"] if bias else []) + ["sg"]
    _check(zip(keys, got, (c[f"{k}_f64"] for k in keys)))


@pytest.mark.parametrize("name", golden_names("layout_"))
def test_layout_conversion_and_formula(name):
    """The component-major / tuple layouts: rows converted to channel-major by the
    package's converters, pushed through the formula and converted back, equal the
    reference's ComponentMajorTensorProduct / TupleTensorProduct values."""
    from ictc_o2_hp_b200 import ComponentMajorTensorProduct
    c = load_golden(name)
    f = _tp_formula(c["channels"], c["m_max"], c["parity"], c["normalization"])
    x, y, w = _t(c["x"], True), _t(c["y"], True), _t(c["w"], True)
    if str(c["cls"]) == "ComponentMajorTensorProduct":
        conv = ComponentMajorTensorProduct(int(c["channels"]), int(c["m_max"]),
                                           parity=str(c["parity"]))
        out = conv._to_component_major(f(conv._to_channel_major(x),
                                          conv._to_channel_major(y), w))
    else:
        # tuple blocks concatenated in block order are the flat channel-major row
        out = f(x, y, w)
    grads = torch.autograd.grad(out, (x, y, w), _t(c["g"]))
    _check(zip(("out", "dx", "dy", "dw"), (out, *grads),
               (c[f"{k}_f64"] for k in ("out", "dx", "dy", "dw"))))
