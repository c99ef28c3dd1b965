"""Second derivatives (force-loss training) of TensorProduct and
UvuTensorProduct through the CUDA kernels, every role at once: the gradients of
<cx, dx> + <cy, dy> + <cw, dw> with respect to x, y, w and the cotangent g,
against the float64 PyTorch formulas on the CPU (the arbiter's role in the
reference, triton_o2.py:1041-1069, uvu_triton.py:442-457), which
tests/test_formula_pins.py pins to the reference's own second derivatives, and
directly against those reference values (tests/golden/second_*.npz); gate 1e-5
normalised max error."""

from __future__ import annotations

import pytest
import torch

from conftest import golden_names, load_golden
from oracle import o2_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _second(fn, x, y, w, g, cot, roles):
    first = torch.autograd.grad(fn(x, y, w), (x, y, w), g, create_graph=True)
    loss = sum((f * c).sum() for f, c in zip(first, cot) if c is not None)
    return torch.autograd.grad(loss, roles, allow_unused=True)


def _check(got, want, names):
    for name, a, b in zip(names, got, want):
        if b is None:
            assert a is None or float(a.abs().max()) == 0.0, name
            continue
        err = O.max_error(a.detach().cpu().double().numpy(), b.detach().numpy())
        assert err <= TOL, f"{name}: {err:.3e}"


def _leaves(*tensors, device=None, dtype=None):
    return tuple(t.detach().to(device=device, dtype=dtype).requires_grad_(True) for t in tensors)


@pytest.mark.parametrize("channels,m_max,parity,rows,present", [
    (8, 2, "full", 37, (1, 1, 1)),
    (5, 3, "canonical", 21, (1, 1, 1)),
    (16, 1, "full", 40, (0, 1, 1)),   # no dx cotangent
    (6, 2, "full", 9, (1, 0, 0)),     # dx cotangent only
])
def test_tensor_product_all_roles(channels, m_max, parity, rows, present, cuda_device):
    from ictc_o2_hp_b200 import TensorProduct
    from ictc_o2_hp_b200.ops import torch_tp_flat
    torch.manual_seed(channels + rows)
    tp = TensorProduct(channels, m_max, parity=parity).to(cuda_device)
    W, n = tp.representation_dimension, tp.weight.numel()
    base = [torch.randn(rows, W), torch.randn(rows, W), torch.randn(n) * 0.1,
            torch.randn(rows, W)]
    cot = [torch.randn(rows, W) if present[0] else None,
           torch.randn(rows, W) if present[1] else None,
           torch.randn(n) if present[2] else None]
    x, y, w, g = _leaves(*base, device=cuda_device)
    got = _second(lambda a, b, c: torch.ops.ictc_o2_b200.tp_forward(a, b, c, channels, m_max,
                                                                      parity, "component"),
                  x, y, w, g, [None if c is None else c.to(cuda_device) for c in cot],
                  (x, y, w, g))
    xc, yc, wc, gc = _leaves(*base, dtype=torch.float64)
    want = _second(lambda a, b, c: torch_tp_flat(a, b, c, tp._plan), xc, yc, wc, gc,
                   [None if c is None else c.double() for c in cot], (xc, yc, wc, gc))
    _check(got, want, ("d x", "d y", "d w", "d g"))


@pytest.mark.parametrize("U,V,m,shared,rows", [
    (16, 8, 2, True, 25),
    (12, 4, 1, False, 13),
    (32, 32, 3, False, 6),
])
def test_uvu_all_roles(U, V, m, shared, rows, cuda_device):
    from ictc_o2_hp_b200 import UvuTensorProduct
    from ictc_o2_hp_b200.ops import torch_uvu_flat
    torch.manual_seed(U + V + rows)
    tp = UvuTensorProduct(U, V, m, shared_weights=shared, internal_weights=False).to(cuda_device)
    n = tp.weight_numel
    wshape = (n,) if shared else (rows, n)
    base = [torch.randn(rows, tp.input1_dimension), torch.randn(rows, tp.input2_dimension),
            torch.randn(*wshape) / V ** 0.5, torch.randn(rows, tp.representation_dimension)]
    cot = [torch.randn(rows, tp.input1_dimension), torch.randn(rows, tp.input2_dimension),
           torch.randn(*wshape)]
    x, y, w, g = _leaves(*base, device=cuda_device)
    got = _second(tp, x, y, w, g, [c.to(cuda_device) for c in cot], (x, y, w, g))
    coef = torch.from_numpy(tp._coefficient_values).double()
    xc, yc, wc, gc = _leaves(*base, dtype=torch.float64)
    want = _second(lambda a, b, c: torch_uvu_flat(a, b, c, tp.entries_in1, tp.entries_in2,
                                                  tp.paths, coef, U, V, shared),
                   xc, yc, wc, gc, [c.double() for c in cot], (xc, yc, wc, gc))
    _check(got, want, ("d x", "d y", "d w", "d g"))


def _second_n(fn, inputs, g, cot, roles):
    first = torch.autograd.grad(fn(*inputs), inputs, g, create_graph=True)
    loss = sum((f * c).sum() for f, c in zip(first, cot))
    return torch.autograd.grad(loss, roles, allow_unused=True)


@pytest.mark.parametrize("U,m,H,bias,rows", [
    (16, 2, 12, True, 30),
    (8, 3, 5, False, 17),
])
def test_radial_all_roles(U, m, H, bias, rows, cuda_device):
    """RadialUvuTensorProduct: second derivatives with respect to x, angular, the
    hidden features, alpha, the bias and g (reference radial_streamed.py:173-207)."""
    from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct
    from ictc_o2_hp_b200.ops import torch_uvu_flat
    torch.manual_seed(U + H + rows)
    tp = UvuTensorProduct(U, 1, m, parity="full", parity_in2="canonical", shared_weights=False)
    model = RadialUvuTensorProduct(tp, torch.nn.Linear(H, tp.weight_numel, bias=bias))
    model = model.to(cuda_device)
    n = tp.weight_numel
    base = [torch.randn(rows, tp.input1_dimension), torch.randn(rows, tp.input2_dimension),
            torch.randn(rows, H), torch.randn(n, H) / H ** 0.5]
    if bias:
        base.append(torch.randn(n) * 0.1)
    g0 = torch.randn(rows, tp.representation_dimension)
    cot = [torch.randn_like(t) for t in base]
    inputs = _leaves(*base, device=cuda_device)
    (g,) = _leaves(g0, device=cuda_device)
    table, rconfig = model.tp._table, model._rconfig()
    empty = inputs[3].new_empty(0)

    def fused(x, y, h, a, b=None):
        return torch.ops.ictc_o2_b200.radial_forward(x, y, h, a, empty if b is None else b,
                                                     table, rconfig, bias)

    got = _second_n(fused, inputs, g, [c.to(cuda_device) for c in cot], (*inputs, g))
    coef = torch.from_numpy(model.tp._coefficient_values).double()
    ref_inputs = _leaves(*base, dtype=torch.float64)
    (gc,) = _leaves(g0, dtype=torch.float64)

    def composed(x, y, h, a, b=None):
        w = h @ a.t() + (0 if b is None else b)
        return torch_uvu_flat(x, y, w, tp.entries_in1, tp.entries_in2, tp.paths, coef, U, 1,
                              False)

    want = _second_n(composed, ref_inputs, gc, [c.double() for c in cot], (*ref_inputs, gc))
    names = ["d x", "d angular", "d hidden", "d alpha"] + (["d bias"] if bias else []) + ["d g"]
    _check(got, want, names)


# ------------------------------------------------ against the reference's own values
# The second derivatives the reference's CPU autograd produced (create_graph) on
# seeded inputs (tests/golden/second_*.npz, written by make_golden.py): the kernels'
# double backward must match them, not only this package's formulas.


def _dev(a, device, grad=True):
    return torch.as_tensor(a, dtype=torch.float32, device=device).requires_grad_(grad)


def _check_fixture(got, case, keys):
    for key, value in zip(keys, got):
        err = O.max_error(value.detach().cpu().double().numpy(), case[f"{key}_f64"])
        assert err <= TOL, f"{key}: {err:.3e}"


@pytest.mark.parametrize("name", golden_names("second_tp_"))
def test_tensor_product_reference_second_order(name, cuda_device):
    from ictc_o2_hp_b200 import TensorProduct
    c = load_golden(name)
    tp = TensorProduct(int(c["channels"]), int(c["m_max"]), parity=str(c["parity"]),
                       normalization=str(c["normalization"])).to(cuda_device)
    with torch.no_grad():
        tp.weight.copy_(torch.as_tensor(c["w"]))
    x, y, g = (_dev(c[k], cuda_device) for k in ("x", "y", "g"))
    got = _second_n(lambda a, b, w: tp(a, b), (x, y, tp.weight), g,
                    [_dev(c[k], cuda_device, False) for k in ("hx", "hy", "hw")],
                    (x, y, tp.weight, g))
    _check_fixture(got, c, ("sx", "sy", "sw", "sg"))


@pytest.mark.parametrize("name", golden_names("second_uvu_"))
def test_uvu_reference_second_order(name, cuda_device):
    from ictc_o2_hp_b200 import UvuTensorProduct
    c = load_golden(name)
    tp = UvuTensorProduct(int(c["u"]), int(c["v"]), int(c["m_max"]),
                          shared_weights=bool(c["shared"]), internal_weights=False)
    tp = tp.to(cuda_device)
    x, y, w, g = (_dev(c[k], cuda_device) for k in ("x", "y", "w", "g"))
    got = _second_n(tp, (x, y, w), g,
                    [_dev(c[k], cuda_device, False) for k in ("hx", "hy", "hw")], (x, y, w, g))
    _check_fixture(got, c, ("sx", "sy", "sw", "sg"))


@pytest.mark.parametrize("name", golden_names("second_radial_"))
def test_radial_reference_second_order(name, cuda_device):
    from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct
    c = load_golden(name)
    bias = bool(c["bias"])
    tp = UvuTensorProduct(int(c["u"]), 1, int(c["m_max"]), parity="full",
                          parity_in2="canonical", shared_weights=False)
    lin = torch.nn.Linear(int(c["hidden"]), tp.weight_numel, bias=bias)
    with torch.no_grad():
        lin.weight.copy_(torch.as_tensor(c["alpha"]))
        if bias:
            lin.bias.copy_(torch.as_tensor(c["b"]))
    model = RadialUvuTensorProduct(tp, lin).to(cuda_device)
    x, y, h, g = (_dev(c[k], cuda_device) for k in ("x", "y", "h", "g"))
    params = (model.radial_out.weight,) + ((model.radial_out.bias,) if bias else ())
    hs = [_dev(c[k], cuda_device, False) for k in ("hx", "hy", "hh", "ha")]
    if bias:
        hs.append(_dev(c["hb"], cuda_device, False))
    operands = (x, y, h, *params)
    got = _second_n(lambda a, b, hh, *p: model(a, b, hh), operands, g, hs, (*operands, g))
    keys = ["sx", "sy", "sh", "sa"] + (["sb"] if bias else []) + ["sg"]
    _check_fixture(got, c, keys)
