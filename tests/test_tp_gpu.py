"""GPU parity of the fused TensorProduct kernels (through the C-ABI) against the
CPU oracle and the reference's golden fixtures.  Gate: normalised max error
max|a-b| / max(1e-7, max|a|, max|b|) <= 1e-5 for out, dx, dy and dw
(the reference's own gate, benchmarks/eqx/scripts/validate_math.py:74)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import o2_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def run_tp(tp, x, y, g, device):
    """fwd + VJP on the GPU; returns numpy (out, dx, dy, dw)."""
    xx = torch.as_tensor(x, dtype=torch.float32, device=device).requires_grad_(True)
    yy = torch.as_tensor(y, dtype=torch.float32, device=device).requires_grad_(True)
    gg = torch.as_tensor(g, dtype=torch.float32, device=device)
    out = tp(xx, yy)
    dx, dy, dw = torch.autograd.grad(out, (xx, yy, tp.weight), gg)
    torch.cuda.synchronize()
    return tuple(t.detach().cpu().numpy() for t in (out, dx, dy, dw))


def make_tp(channels, m_max, parity, normalization, weight, device):
    from ictc_o2_hp_b200 import TensorProduct
    tp = TensorProduct(channels, m_max, parity=parity, normalization=normalization).to(device)
    with torch.no_grad():
        tp.weight.copy_(torch.as_tensor(weight))
    return tp


def assert_close(got, want, tol=TOL):
    for name, a, b in zip(("out", "dx", "dy", "dw"), got, want):
        err = O.max_error(a, b)
        assert err <= tol, f"{name}: normalised error {err:.3e} > {tol}"


@pytest.mark.parametrize("name", [n for n in golden_names("tp_") if "cfg" not in n])
def test_golden_fixtures(name, cuda_device):
    case = load_golden(name)
    tp = make_tp(int(case["channels"]), int(case["m_max"]), str(case["parity"]),
                 str(case["normalization"]), case["weight"], cuda_device)
    got = run_tp(tp, case["x"], case["y"], case["g"], cuda_device)
    assert_close(got, tuple(case[f"{k}_f64"] for k in ("out", "dx", "dy", "dw")))


def _replay(case):
    import torch as T
    oracle = O.TpOracle(int(case["channels"]), int(case["m_max"]), str(case["parity"]),
                        str(case["normalization"]))
    T.manual_seed(int(case["seed"]))
    for (_, _, _, s, e, _, _) in oracle.paths:
        T.randn(e - s)
    rows = int(case["torch_rows"])
    return T.randn(rows, oracle.width), T.randn(rows, oracle.width)


@pytest.mark.parametrize("name", ["tp_c32_m2_canonical_cfg1", "tp_c128_m6_full_cfg2"])
def test_benchmark_recipe_full_size(name, cuda_device):
    """Configs 1 and 2 exactly as the benchmark defines them (seeded init, iid
    N(0,1) inputs, ones cotangent), at their full N, against the reference's f64
    values: sampled rows, per-column sums over all rows, and the whole dw."""
    case = load_golden(name)
    x, y = _replay(case)
    tp = make_tp(int(case["channels"]), int(case["m_max"]), str(case["parity"]),
                 str(case["normalization"]), case["weight"], cuda_device)
    out, dx, dy, dw = run_tp(tp, x, y, torch.ones_like(x), cuda_device)
    rows = case["keep_rows"]
    for key, value in (("out", out), ("dx", dx), ("dy", dy)):
        assert O.max_error(value[rows], case[f"{key}_f64_rows"]) <= TOL, key
        assert O.max_error(value.astype(np.float64).sum(axis=0),
                           case[f"{key}_f64_sum"]) <= TOL, key
    assert O.max_error(dw, case["dw_f64"]) <= TOL


SHAPES = [
    # (channels, m_max, parity, normalization, rows)
    (32, 2, "canonical", "component", 257),
    (128, 6, "full", "component", 64),
    (64, 3, "full", "component", 300),
    (96, 4, "canonical", "component", 65),
    (256, 6, "full", "component", 9),
    (17, 3, "full", "norm", 45),
    (33, 5, "canonical", "norm", 31),
    (1, 0, "full", "component", 7),
    (1, 1, "canonical", "component", 3),
    (5, 7, "full", "component", 11),
    (3, 8, "canonical", "norm", 6),
    (48, 1, "full", "component", 1000),
    # channel-tiled backward (more channel groups than a staged CTA holds, m_max >= 3:
    # tiles of 64 / 128 channels) and the shapes next to it that keep the untiled kernels
    (96, 3, "full", "component", 300),
    (192, 4, "full", "component", 21),
    (256, 3, "full", "norm", 33),
    (256, 2, "full", "component", 13),
    (320, 3, "canonical", "component", 40),
]


@pytest.mark.parametrize("channels,m_max,parity,normalization,rows", SHAPES)
def test_against_oracle(channels, m_max, parity, normalization, rows, cuda_device):
    oracle = O.TpOracle(channels, m_max, parity, normalization)
    rng = np.random.default_rng(channels * 1000 + m_max * 10 + rows)
    x = rng.standard_normal((rows, oracle.width)).astype(np.float32)
    y = rng.standard_normal((rows, oracle.width)).astype(np.float32)
    g = rng.standard_normal((rows, oracle.width)).astype(np.float32)
    w = (rng.standard_normal(oracle.weight_numel) * 0.5).astype(np.float32)
    want = oracle.vjp(*(a.astype(np.float64) for a in (x, y, w, g)))
    tp = make_tp(channels, m_max, parity, normalization, w, cuda_device)
    assert_close(run_tp(tp, x, y, g, cuda_device), want)


def test_empty_rows(cuda_device):
    from ictc_o2_hp_b200 import TensorProduct
    tp = TensorProduct(8, 2).to(cuda_device)
    x = torch.zeros(0, tp.representation_dimension, device=cuda_device, requires_grad=True)
    out = tp(x, x)
    assert out.shape == x.shape
    dx, dw = torch.autograd.grad(out, (x, tp.weight), torch.zeros_like(out))
    assert dx.shape == x.shape and torch.count_nonzero(dw) == 0


def test_batch_shape_and_noncontiguous(cuda_device):
    """(*batch, W) inputs and a strided view, compared with contiguous flat rows."""
    from ictc_o2_hp_b200 import TensorProduct
    torch.manual_seed(1)
    tp = TensorProduct(16, 3).to(cuda_device)
    W = tp.representation_dimension
    x = torch.randn(4, 5, W, device=cuda_device)
    y = torch.randn(4, 5, W, device=cuda_device)
    out = tp(x, y)
    assert out.shape == (4, 5, W)
    flat = tp(x.reshape(-1, W), y.reshape(-1, W)).reshape(4, 5, W)
    assert torch.equal(out, flat)
    big = torch.randn(20, 2 * W, device=cuda_device)
    view = big[:, :W]  # strided rows
    assert torch.equal(tp(view, y.reshape(-1, W)), tp(view.contiguous(), y.reshape(-1, W)))


def test_unaligned_operands_take_scalar_path(cuda_device):
    """Odd-width canonical rows (C odd) are 4-byte aligned only; results still match."""
    oracle = O.TpOracle(7, 2, "canonical")
    rng = np.random.default_rng(5)
    x, y, g = (rng.standard_normal((13, oracle.width)).astype(np.float32) for _ in range(3))
    w = rng.standard_normal(oracle.weight_numel).astype(np.float32)
    tp = make_tp(7, 2, "canonical", "component", w, cuda_device)
    assert_close(run_tp(tp, x, y, g, cuda_device),
                 oracle.vjp(*(a.astype(np.float64) for a in (x, y, w, g))))


def test_deterministic_weight_gradient(cuda_device):
    from ictc_o2_hp_b200 import TensorProduct
    torch.manual_seed(2)
    tp = TensorProduct(128, 6).to(cuda_device)
    x = torch.randn(4099, tp.representation_dimension, device=cuda_device)
    y = torch.randn_like(x)
    g = torch.randn_like(x)
    results = []
    for _ in range(2):
        xx, yy = x.clone().requires_grad_(True), y.clone().requires_grad_(True)
        results.append(torch.autograd.grad(tp(xx, yy), (xx, yy, tp.weight), g))
    for a, b in zip(*results):
        assert torch.equal(a, b)


def test_bilinearity_at_full_size(cuda_device):
    """TP(x, y1 + y2) = TP(x, y1) + TP(x, y2) at the config-2 size."""
    from ictc_o2_hp_b200 import TensorProduct
    torch.manual_seed(3)
    tp = TensorProduct(128, 6).to(cuda_device)
    x = torch.randn(65536, tp.representation_dimension, device=cuda_device)
    y1, y2 = torch.randn_like(x), torch.randn_like(x)
    with torch.no_grad():
        lhs = tp(x, y1 + y2)
        rhs = tp(x, y1) + tp(x, y2)
    assert O.max_error(lhs.cpu().numpy(), rhs.cpu().numpy()) < 1e-5


def test_torch_compile_fullgraph(cuda_device):
    from ictc_o2_hp_b200 import TensorProduct
    torch.manual_seed(4)
    tp = TensorProduct(64, 4).to(cuda_device)
    x = torch.randn(640, tp.representation_dimension, device=cuda_device, requires_grad=True)
    y = torch.randn_like(x, requires_grad=True)
    compiled = torch.compile(tp, fullgraph=True, dynamic=False)
    out = compiled(x, y)
    grads = torch.autograd.grad(out, (x, y, tp.weight), torch.ones_like(out))
    ref = tp(x, y)
    ref_grads = torch.autograd.grad(ref, (x, y, tp.weight), torch.ones_like(ref))
    assert torch.equal(out, ref)
    for a, b in zip(grads, ref_grads):
        assert torch.equal(a, b)


def test_double_backward_matches_formula(cuda_device):
    """Second derivatives (PyTorch recomputation on the GPU) against the same
    formula evaluated in float64 on the CPU."""
    from ictc_o2_hp_b200 import TensorProduct
    from ictc_o2_hp_b200.ops import torch_tp_flat
    torch.manual_seed(5)
    tp = TensorProduct(8, 3).to(cuda_device)
    W = tp.representation_dimension
    x = torch.randn(6, W, device=cuda_device, requires_grad=True)
    y = torch.randn(6, W, device=cuda_device, requires_grad=True)
    g = torch.randn(6, W, device=cuda_device)
    dx, = torch.autograd.grad(tp(x, y), (x,), g, create_graph=True)
    second = torch.autograd.grad(dx.square().sum(), (y, tp.weight))
    xc, yc = x.detach().cpu().double().requires_grad_(), y.detach().cpu().double().requires_grad_()
    wc = tp.weight.detach().cpu().double().requires_grad_()
    dxc, = torch.autograd.grad(torch_tp_flat(xc, yc, wc, tp._plan), (xc,), g.cpu().double(),
                               create_graph=True)
    want = torch.autograd.grad(dxc.square().sum(), (yc, wc))
    for a, b in zip(second, want):
        assert O.max_error(a.cpu().numpy(), b.numpy()) <= TOL


def test_tuple_and_component_major_layouts(cuda_device):
    from ictc_o2_hp_b200 import ComponentMajorTensorProduct, TensorProduct, TupleTensorProduct
    torch.manual_seed(6)
    flat = TensorProduct(12, 3).to(cuda_device)
    tup = TupleTensorProduct(12, 3).to(cuda_device)
    comp = ComponentMajorTensorProduct(12, 3).to(cuda_device)
    for m in (tup, comp):
        m.load_state_dict(flat.state_dict())
    W = flat.representation_dimension
    x, y = torch.randn(10, W, device=cuda_device), torch.randn(10, W, device=cuda_device)
    ref = flat(x, y)
    split = lambda v: tuple(  # noqa: E731
        v[:, o:o + b.multiplicity * b.irrep_dimension].reshape(10, b.multiplicity,
                                                                b.irrep_dimension)
        for b, o in zip(flat.blocks, flat._plan.key_offsets().values()))
    got = torch.cat([t.reshape(10, -1) for t in tup(split(x), split(y))], dim=-1)
    assert torch.equal(got, ref)
    cm = comp(comp._to_component_major(x), comp._to_component_major(y))
    assert torch.equal(comp._to_channel_major(cm), ref)


@pytest.mark.parametrize("channels,m_max,parity,rows,variant", [
    (16, 3, "full", 300, None),
    (12, 2, "canonical", 77, None),
    (128, 6, "full", 2048, None),      # the benchmark configuration's width (staged kernels)
    (9, 4, "full", 50, "direct"),      # odd channel count, direct kernels
    (32, 2, "full", 640, "grouped"),
    (256, 3, "full", 200, None),       # channel-tiled backward
    (128, 6, "full", 1001, "widepair"),  # row-paired wide forward, odd row count
])
def test_component_major_in_place(channels, m_max, parity, rows, variant, cuda_device,
                                  monkeypatch):
    """ComponentMajorTensorProduct reads and writes component-major rows in place
    (ICTC_LAYOUT_COMPONENT_MAJOR): forward, dx, dy, dw and the second derivatives
    equal the channel-major product on the converted rows, bit for bit."""
    from ictc_o2_hp_b200 import ComponentMajorTensorProduct, TensorProduct
    if variant:
        monkeypatch.setenv("ICTC_TP_FORWARD", variant)
    torch.manual_seed(channels + rows)
    flat = TensorProduct(channels, m_max, parity=parity).to(cuda_device)
    comp = ComponentMajorTensorProduct(channels, m_max, parity=parity).to(cuda_device)
    comp.load_state_dict(flat.state_dict())
    W = flat.representation_dimension
    x, y, g = (torch.randn(rows, W, device=cuda_device) for _ in range(3))
    xc, yc, gc = (comp._to_component_major(t) for t in (x, y, g))
    xf, yf = x.clone().requires_grad_(True), y.clone().requires_grad_(True)
    xm, ym = xc.clone().requires_grad_(True), yc.clone().requires_grad_(True)
    ref = flat(xf, yf)
    got = comp(xm, ym)
    assert torch.equal(comp._to_channel_major(got), ref)
    rf = torch.autograd.grad(ref, (xf, yf, flat.weight), g, create_graph=True)
    rm = torch.autograd.grad(got, (xm, ym, comp.weight), gc, create_graph=True)
    assert torch.equal(comp._to_channel_major(rm[0]), rf[0])
    assert torch.equal(comp._to_channel_major(rm[1]), rf[1])
    assert torch.equal(rm[2], rf[2])
    # second derivatives: d/d(x, y) of <dx, cot>
    cot = torch.randn(rows, W, device=cuda_device)
    sf = torch.autograd.grad((rf[0] * cot).sum(), (yf, flat.weight))
    sm = torch.autograd.grad((rm[0] * comp._to_component_major(cot)).sum(), (ym, comp.weight))
    assert torch.equal(comp._to_channel_major(sm[0]), sf[0])
    assert torch.equal(sm[1], sf[1])


@pytest.mark.parametrize("channels,m_max,parity,rows", [
    (128, 6, "full", 333),       # the benchmark configuration's width, odd row count
    (32, 4, "canonical", 1001),  # four rows per stage block
    (96, 5, "full", 64),         # six channel groups
    (64, 6, "canonical", 4097),
])
def test_row_paired_wide_forward_matches_wide(channels, m_max, parity, rows, cuda_device,
                                              monkeypatch):
    """The row-paired wide forward (ICTC_TP_FORWARD=widepair: two rows per warp as the
    halves of paired f32x2 operations) is bit-identical to the wide forward."""
    from ictc_o2_hp_b200 import TensorProduct, _lib
    torch.manual_seed(channels + rows)
    tp = TensorProduct(channels, m_max, parity=parity).to(cuda_device)
    x = torch.randn(rows, tp.representation_dimension, device=cuda_device)
    y = torch.randn_like(x)
    with torch.no_grad():
        monkeypatch.setenv("ICTC_TP_FORWARD", "wide")
        ref = tp(x, y)
        monkeypatch.setenv("ICTC_TP_FORWARD", "widepair")
        got = tp(x, y)
    assert torch.equal(got, ref)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("variant", ["staged", "wide", "direct", "grouped", "widepair"])
def test_forward_variants_agree(variant, cuda_device, monkeypatch):
    """Every forward kernel selectable with ICTC_TP_FORWARD (staged ring, wide
    staged, register-weight direct, shared-weight grouped) gives the same values
    as the default choice."""
    from ictc_o2_hp_b200 import TensorProduct
    torch.manual_seed(7)
    for channels, m_max, parity in ((128, 6, "full"), (32, 2, "canonical"), (48, 3, "full")):
        tp = TensorProduct(channels, m_max, parity=parity).to(cuda_device)
        x = torch.randn(333, tp.representation_dimension, device=cuda_device)
        y = torch.randn_like(x)
        with torch.no_grad():
            ref = tp(x, y)
            monkeypatch.setenv("ICTC_TP_FORWARD", variant)
            got = tp(x, y)
            monkeypatch.delenv("ICTC_TP_FORWARD")
        assert O.max_error(got.cpu().numpy(), ref.cpu().numpy()) < 1e-6


def test_no_device_error_flag(cuda_device):
    from ictc_o2_hp_b200 import _lib
    assert _lib.device_error() == 0



@pytest.mark.parametrize("name", golden_names("layout_"))
def test_layout_classes_against_reference(name, cuda_device):
    """ComponentMajorTensorProduct and TupleTensorProduct against the values of the
    reference's own classes of the same name (api.py:32-49), forward and VJP."""
    import ictc_o2_hp_b200 as P
    c = load_golden(name)
    cls = getattr(P, str(c["cls"]))
    tp = cls(int(c["channels"]), int(c["m_max"]), parity=str(c["parity"]),
             normalization=str(c["normalization"])).to(cuda_device)
    with torch.no_grad():
        tp.weight.copy_(torch.as_tensor(c["w"]))
    x, y = (torch.as_tensor(c[k], device=cuda_device).requires_grad_(True) for k in ("x", "y"))
    g = torch.as_tensor(c["g"], device=cuda_device)
    if str(c["cls"]) == "TupleTensorProduct":
        rows = x.shape[0]

        def split(v):
            parts, cursor = [], 0
            for b in tp.blocks:
                width = b.multiplicity * b.irrep_dimension
                parts.append(v[:, cursor:cursor + width].reshape(rows, b.multiplicity,
                                                                 b.irrep_dimension))
                cursor += width
            return tuple(parts)
        out = torch.cat([t.reshape(rows, -1) for t in tp(split(x), split(y))], dim=-1)
    else:
        out = tp(x, y)
    grads = torch.autograd.grad(out, (x, y, tp.weight), g)
    got = tuple(t.detach().cpu().numpy() for t in (out, *grads))
    assert_close(got, tuple(c[f"{k}_f64"] for k in ("out", "dx", "dy", "dw")))


@pytest.mark.parametrize("channels,m_max,parity,rows", [
    (256, 6, "full", 333),
    (192, 3, "full", 70),
    (320, 4, "canonical", 129),
])
def test_tiled_backward_matches_untiled(channels, m_max, parity, rows, cuda_device, monkeypatch):
    """The channel-tiled backward (ICTC_TP_BACKWARD unset or "tiled") against the
    untiled kernels on the same rows: dx and dy bit for bit (the same per-row
    arithmetic), dw to float32 summation-order differences."""
    from ictc_o2_hp_b200 import TensorProduct
    torch.manual_seed(channels + rows)
    tp = TensorProduct(channels, m_max, parity=parity).to(cuda_device)
    W = tp.representation_dimension
    x, y, g = (torch.randn(rows, W, device=cuda_device) for _ in range(3))
    w = tp.weight.detach()
    args = (channels, m_max, parity, "component")
    tiled = torch.ops.ictc_o2_b200.tp_backward(x, y, w, g, *args)
    monkeypatch.setenv("ICTC_TP_BACKWARD", "untiled")
    plain = torch.ops.ictc_o2_b200.tp_backward(x, y, w, g, *args)
    assert torch.equal(tiled[0], plain[0]) and torch.equal(tiled[1], plain[1])
    assert O.max_error(tiled[2].cpu().numpy(), plain[2].cpu().numpy()) < 1e-6


@pytest.mark.parametrize("channels,m_max,parity,rows", [
    (128, 2, "full", 4000),
    (96, 3, "full", 3001),
    (96, 2, "canonical", 5000),
    (64, 1, "canonical", 777),
])
def test_paired_staged_backward_matches_single(channels, m_max, parity, rows, cuda_device,
                                               monkeypatch):
    """Small orders run two staged-backward CTAs per SM (registers permitting, half the
    stage ring each); against one CTA per SM (ICTC_TP_BACKWARD_PAIRS=0) on the same rows:
    dx and dy bit for bit, dw to float32 summation-order differences (twice the slots)."""
    from ictc_o2_hp_b200 import TensorProduct
    torch.manual_seed(channels + rows)
    tp = TensorProduct(channels, m_max, parity=parity).to(cuda_device)
    W = tp.representation_dimension
    x, y, g = (torch.randn(rows, W, device=cuda_device) for _ in range(3))
    w = tp.weight.detach()
    args = (channels, m_max, parity, "component")
    paired = torch.ops.ictc_o2_b200.tp_backward(x, y, w, g, *args)
    monkeypatch.setenv("ICTC_TP_BACKWARD_PAIRS", "0")
    single = torch.ops.ictc_o2_b200.tp_backward(x, y, w, g, *args)
    assert torch.equal(paired[0], single[0]) and torch.equal(paired[1], single[1])
    assert O.max_error(paired[2].cpu().numpy(), single[2].cpu().numpy()) < 1e-6


@pytest.mark.parametrize("channels,m_max,parity,rows", [
    (128, 3, "full", 4001),    # odd: the last warp pair has one row
    (64, 4, "full", 3000),
    (32, 3, "full", 777),
])
def test_row_paired_backward_matches_scalar(channels, m_max, parity, rows, cuda_device,
                                            monkeypatch):
    """Full parity at m_max 3-4 runs the row-paired staged backward (two rows per warp in
    paired f32x2 arithmetic); against the scalar staged kernel (ICTC_TP_BACKWARD_ROWPAIR=0)
    on the same rows: dx and dy bit for bit, dw to float32 summation-order differences."""
    from ictc_o2_hp_b200 import TensorProduct
    torch.manual_seed(channels + rows)
    tp = TensorProduct(channels, m_max, parity=parity).to(cuda_device)
    W = tp.representation_dimension
    x, y, g = (torch.randn(rows, W, device=cuda_device) for _ in range(3))
    w = tp.weight.detach()
    args = (channels, m_max, parity, "component")
    paired = torch.ops.ictc_o2_b200.tp_backward(x, y, w, g, *args)
    monkeypatch.setenv("ICTC_TP_BACKWARD_ROWPAIR", "0")
    scalar = torch.ops.ictc_o2_b200.tp_backward(x, y, w, g, *args)
    assert torch.equal(paired[0], scalar[0]) and torch.equal(paired[1], scalar[1])
    assert O.max_error(paired[2].cpu().numpy(), scalar[2].cpu().numpy()) < 1e-6
