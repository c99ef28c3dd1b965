"""GPU parity of the uvu kernels (through the C-ABI) against the reference's golden
fixtures and the CPU oracle; gate 1e-5 normalised max error."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import o2_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def run(tp, x, y, w, g, device, shared):
    xx = torch.as_tensor(x, dtype=torch.float32, device=device).requires_grad_(True)
    yy = torch.as_tensor(y, dtype=torch.float32, device=device).requires_grad_(True)
    ww = torch.as_tensor(w, dtype=torch.float32, device=device).requires_grad_(True)
    out = tp(xx, yy, ww)
    grads = torch.autograd.grad(out, (xx, yy, ww), torch.as_tensor(g, device=device))
    torch.cuda.synchronize()
    return (out.detach().cpu().numpy(), *(t.cpu().numpy() for t in grads))


def check(got, want):
    for name, a, b in zip(("out", "dx", "dy", "dw"), got, want):
        err = O.max_error(a, b)
        assert err <= TOL, f"{name}: {err:.3e}"


@pytest.mark.parametrize("name", golden_names("uvu_"))
def test_golden(name, cuda_device):
    from ictc_o2_hp_b200 import UvuTensorProduct
    c = load_golden(name)
    shared = bool(c["shared"])
    tp = UvuTensorProduct(int(c["u"]), int(c["v"]), int(c["m_max"]), parity=str(c["parity"]),
                          parity_in2=str(c["parity_in2"]), m_max_in2=int(c["m_max_in2"]),
                          normalization=str(c["normalization"]),
                          path_normalization=str(c["path_normalization"]),
                          shared_weights=shared, internal_weights=False).to(cuda_device)
    got = run(tp, c["x"], c["y"], c["w"], c["g"], cuda_device, shared)
    check(got, tuple(c[f"{k}_f64"] for k in ("out", "dx", "dy", "dw")))


CASES = [
    # U, V, m1, parity, m2, parity2, norm, pnorm, shared, rows
    (128, 32, 3, "full", 3, "full", "component", "none", True, 70),   # config 4, shared
    (128, 32, 3, "full", 3, "full", "component", "none", False, 9),   # config 4, per row
    (64, 1, 3, "full", 3, "canonical", "component", "none", False, 40),  # radial shape
    (33, 7, 2, "canonical", 3, "full", "norm", "path", True, 45),
    (130, 40, 1, "full", 1, "full", "component", "none", True, 33),   # U > 128, V > 32
    (5, 3, 4, "full", 2, "canonical", "component", "element", True, 65),
    (1, 1, 0, "full", 0, "full", "component", "none", True, 3),
    (16, 8, 2, "canonical", 2, "full", "component", "none", False, 21),   # streamed per row
    (200, 16, 1, "full", 1, "full", "norm", "none", False, 5),       # two channel chunks
    (96, 64, 2, "full", 1, "canonical", "component", "path", False, 4),  # V = 64
    (8, 4, 1, "full", 3, "full", "component", "none", True, 50),  # second entries no path reads
    (8, 4, 1, "full", 3, "full", "component", "none", False, 20),  # the same, per-row weights
    (128, 32, 3, "full", 3, "full", "component", "none", True, 520),  # two dw row chunks
]


@pytest.mark.parametrize("case", CASES)
def test_against_oracle(case, cuda_device):
    from ictc_o2_hp_b200 import UvuTensorProduct
    U, V, m1, p1, m2, p2, norm, pnorm, shared, rows = case
    oracle = O.UvuOracle(U, V, m1, p1, p2, m2, norm, pnorm)
    tp = UvuTensorProduct(U, V, m1, parity=p1, m_max_in2=m2, parity_in2=p2,
                          normalization=norm, path_normalization=pnorm,
                          shared_weights=shared, internal_weights=False).to(cuda_device)
    rng = np.random.default_rng(U * 100 + V + rows)
    x = rng.standard_normal((rows, tp.input1_dimension)).astype(np.float32)
    y = rng.standard_normal((rows, tp.input2_dimension)).astype(np.float32)
    wshape = (tp.weight_numel,) if shared else (rows, tp.weight_numel)
    w = (rng.standard_normal(wshape) / np.sqrt(V)).astype(np.float32)
    g = rng.standard_normal((rows, tp.representation_dimension)).astype(np.float32)
    want = oracle.vjp(*(a.astype(np.float64) for a in (x, y, w, g)), shared=shared)
    check(run(tp, x, y, w, g, cuda_device, shared), want)


@pytest.mark.parametrize("case", [c for c in CASES if c[8]][:3])
def test_split_thread_tile(case, cuda_device, monkeypatch):
    """Shared-weight forward / dx with the 4 x 8 per-thread tile (ICTC_UVU_TILE=split);
    the default 4 x 4 tile runs every other case."""
    monkeypatch.setenv("ICTC_UVU_TILE", "split")
    test_against_oracle(case, cuda_device)


def test_role_pruning_and_empty(cuda_device):
    from ictc_o2_hp_b200 import UvuTensorProduct
    torch.manual_seed(0)
    tp = UvuTensorProduct(16, 4, 2).to(cuda_device)
    x = torch.randn(20, tp.input1_dimension, device=cuda_device, requires_grad=True)
    y = torch.randn(20, tp.input2_dimension, device=cuda_device)
    out = tp(x, y)
    dx, dw = torch.autograd.grad(out.square().sum(), (x, tp.weight))
    xx = x.detach().requires_grad_(True)
    yy = y.clone().requires_grad_(True)
    ref = torch.autograd.grad(tp(xx, yy).square().sum(), (xx, yy, tp.weight))
    assert torch.allclose(dx, ref[0]) and torch.allclose(dw, ref[2])
    empty = torch.zeros(0, tp.input1_dimension, device=cuda_device, requires_grad=True)
    e_out = tp(empty, torch.zeros(0, tp.input2_dimension, device=cuda_device))
    (gw,) = torch.autograd.grad(e_out.sum(), (tp.weight,))
    assert e_out.shape == (0, tp.input1_dimension) and torch.count_nonzero(gw) == 0


def test_compile_and_double_backward(cuda_device):
    from ictc_o2_hp_b200 import UvuTensorProduct
    from ictc_o2_hp_b200.ops import torch_uvu_flat
    torch.manual_seed(1)
    tp = UvuTensorProduct(8, 3, 2).to(cuda_device)
    x = torch.randn(12, tp.input1_dimension, device=cuda_device, requires_grad=True)
    y = torch.randn(12, tp.input2_dimension, device=cuda_device, requires_grad=True)
    compiled = torch.compile(tp, fullgraph=True, dynamic=False)
    out = compiled(x, y)
    assert torch.equal(out, tp(x, y))
    (dx,) = torch.autograd.grad(tp(x, y).square().sum(), (x,), create_graph=True)
    second = torch.autograd.grad(dx.sum(), (y, tp.weight))
    coef = torch.from_numpy(tp._coefficient_values)
    xc, yc = x.detach().cpu().double().requires_grad_(), y.detach().cpu().double().requires_grad_()
    wc = tp.weight.detach().cpu().double().requires_grad_()
    val = torch_uvu_flat(xc, yc, wc, tp.entries_in1, tp.entries_in2, tp.paths, coef, 8, 3, True)
    (dxc,) = torch.autograd.grad(val.square().sum(), (xc,), create_graph=True)
    want = torch.autograd.grad(dxc.sum(), (yc, wc))
    for a, b in zip(second, want):
        assert O.max_error(a.cpu().numpy(), b.numpy()) <= TOL


# Per-row-weight cases, each run on every per-row kernel the C-ABI can pick:
# "quad" (V in {8, 16, 32, 64}), "stream" (V a multiple of 8) and "rowwise"
# (any shape); a kernel that does not fit the shape hands over to the next.
PER_ROW = [c for c in CASES if not c[8]] + [
    (160, 32, 1, "full", 1, "full", "component", "none", False, 6),  # two channel chunks
    (64, 16, 2, "full", 2, "full", "norm", "path", False, 7),
]
ROW_KERNELS = ["quad", "stream", "rowwise"]


@pytest.mark.parametrize("kernel", ROW_KERNELS)
@pytest.mark.parametrize("case", PER_ROW)
def test_per_row_kernels(kernel, case, cuda_device, monkeypatch):
    monkeypatch.setenv("ICTC_UVU_ROW_KERNEL", kernel)
    test_against_oracle(case, cuda_device)


@pytest.mark.parametrize("kernel", ROW_KERNELS)
@pytest.mark.parametrize("U,V", [(32, 8), (128, 32), (96, 64)])
def test_per_row_role_pruning(kernel, U, V, cuda_device, monkeypatch):
    """Per-row weights: each subset of requested gradients equals the full VJP."""
    from ictc_o2_hp_b200 import UvuTensorProduct
    monkeypatch.setenv("ICTC_UVU_ROW_KERNEL", kernel)
    torch.manual_seed(3)
    tp = UvuTensorProduct(U, V, 2, shared_weights=False).to(cuda_device)
    x = torch.randn(11, tp.input1_dimension, device=cuda_device, requires_grad=True)
    y = torch.randn(11, tp.input2_dimension, device=cuda_device, requires_grad=True)
    w = torch.randn(11, tp.weight_numel, device=cuda_device, requires_grad=True)
    full = torch.autograd.grad(tp(x, y, w).square().sum(), (x, y, w))
    for i, t in enumerate((x, y, w)):
        (only,) = torch.autograd.grad(tp(x, y, w).square().sum(), (t,))
        assert torch.equal(only, full[i])
