"""Benchmark configs 4 and 5 at their full sizes against the reference's float64
values: UvuTensorProduct(128, 32, 3) with shared weights over 131,072 rows, with
per-row weights over 16,384 rows, and the config-5 radial layer over 1,048,576
edges.  The fixtures hold what the reference's CPU path computed on the same seeded
inputs (tests/golden/make_golden.py over tests/golden/recipes.py, which these tests
use to rebuild the inputs): sampled rows, per-column sums over all rows and, for the
cross-row reductions, the whole weight gradient (uvu dw; radial dalpha and dbias),
the pattern of the reference's own validator (benchmarks/eqx/scripts/
validate_math.py:54-74).  The per-row case also checks every row against the
float64 PyTorch formula on the GPU (pinned to the reference in
tests/test_formula_pins.py).  Gate: max|a-b| / max(1e-7, max|a|, max|b|) <= 1e-5."""

from __future__ import annotations

import math
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden
from oracle import o2_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5

if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))
import recipes as R  # noqa: E402


def _column_sums(t: torch.Tensor, chunk: int = 65536) -> np.ndarray:
    total = torch.zeros(t.shape[1], dtype=torch.float64, device=t.device)
    for s in range(0, t.shape[0], chunk):
        total += t[s:s + chunk].double().sum(0)
    return total.cpu().numpy()


def _check_rows_sums(values: dict, case: dict, keep):
    idx = torch.as_tensor(np.asarray(keep), device=next(iter(values.values())).device)
    for key, value in values.items():
        rows = value.index_select(0, idx).cpu().double().numpy()
        err = O.max_error(rows, case[f"{key}_f64_rows"])
        assert err <= TOL, f"{key} rows: {err:.3e}"
        err = O.max_error(_column_sums(value), case[f"{key}_f64_sum"])
        assert err <= TOL, f"{key} column sums: {err:.3e}"


def test_uvu_config4_shared_full(cuda_device):
    from ictc_o2_hp_b200 import UvuTensorProduct
    case = load_golden("full_uvu_cfg4_shared")
    c = R.CFG4
    x, y, w, g = (torch.from_numpy(a).to(cuda_device) for a in R.cfg4_shared_inputs())
    tp = UvuTensorProduct(c["u"], c["v"], c["m_max"], shared_weights=True,
                          internal_weights=False).to(cuda_device)
    x.requires_grad_(True), y.requires_grad_(True), w.requires_grad_(True)
    out = tp(x, y, w)
    dx, dy, dw = torch.autograd.grad(out, (x, y, w), g)
    torch.cuda.synchronize()
    _check_rows_sums({"out": out.detach(), "dx": dx, "dy": dy}, case, case["keep_rows"])
    err = O.max_error(dw.cpu().double().numpy(), case["dw_f64"])
    assert err <= TOL, f"dw: {err:.3e}"


class _ErrorAccumulator:
    """max|a-b| and max(|a|, |b|) over chunks, for the normalised error of a
    tensor compared piecewise."""

    def __init__(self):
        self.diff, self.scale = 0.0, 1e-7

    def add(self, got: torch.Tensor, want: torch.Tensor):
        got = got.double()
        self.diff = max(self.diff, float((got - want).abs().max()))
        self.scale = max(self.scale, float(got.abs().max()), float(want.abs().max()))

    @property
    def error(self):
        return self.diff / self.scale


def test_uvu_config4_per_row_full(cuda_device):
    """Per-row weights over 16,384 rows (a 39.7 GB weight tensor and as large a
    gradient).  Sampled rows take their inputs from their own seeded numpy streams
    and are checked against the reference's values; the other rows are filled on
    the GPU, and every row is checked against the float64 formula in chunks."""
    from ictc_o2_hp_b200 import UvuTensorProduct
    from ictc_o2_hp_b200.ops import torch_uvu_flat
    case = load_golden("full_uvu_cfg4_perrow_rows")
    c = R.CFG4
    n = R.CFG4_PERROW_ROWS
    gen = torch.Generator(device=cuda_device)
    gen.manual_seed(R.CFG4_PERROW_SEED)
    x = torch.randn(n, c["width1"], device=cuda_device, generator=gen)
    y = torch.randn(n, c["width2"], device=cuda_device, generator=gen)
    g = torch.randn(n, c["width1"], device=cuda_device, generator=gen)
    w = torch.empty(n, c["weight_numel"], device=cuda_device)
    for s in range(0, n, 1024):
        w[s:s + 1024].normal_(generator=gen).mul_(1 / math.sqrt(c["v"]))
    keep = list(R.CFG4_PERROW_KEEP)
    for r in keep:
        for dst, src in zip((x, y, w, g), R.cfg4_perrow_row(r)):
            dst[r].copy_(torch.from_numpy(src))
    tp = UvuTensorProduct(c["u"], c["v"], c["m_max"], shared_weights=False,
                          internal_weights=False).to(cuda_device)
    x.requires_grad_(True), y.requires_grad_(True), w.requires_grad_(True)
    out = tp(x, y, w)
    dx, dy, dw = torch.autograd.grad(out, (x, y, w), g)
    torch.cuda.synchronize()
    idx = torch.as_tensor(keep, device=cuda_device)
    cols = torch.as_tensor(case["dw_columns"], device=cuda_device)
    for key, value in (("out", out.detach()), ("dx", dx), ("dy", dy),
                       ("dw", dw.index_select(1, cols))):
        err = O.max_error(value.index_select(0, idx).cpu().double().numpy(), case[f"{key}_f64"])
        assert err <= TOL, f"{key} sampled rows: {err:.3e}"
    x, y, w = x.detach(), y.detach(), w.detach()
    out = out.detach()
    coef = torch.from_numpy(tp._coefficient_values).double().to(cuda_device)
    acc = {k: _ErrorAccumulator() for k in ("out", "dx", "dy", "dw")}
    chunk = 256
    for s in range(0, n, chunk):
        sl = slice(s, s + chunk)
        xc, yc, wc = (t[sl].double().requires_grad_(True) for t in (x, y, w))
        ref = torch_uvu_flat(xc, yc, wc, tp.entries_in1, tp.entries_in2, tp.paths, coef,
                             c["u"], c["v"], False)
        grads = torch.autograd.grad(ref, (xc, yc, wc), g[sl].double())
        for key, got, want in zip(("out", "dx", "dy", "dw"), (out[sl], dx[sl], dy[sl], dw[sl]),
                                  (ref.detach(), *grads)):
            acc[key].add(got, want)
        del xc, yc, wc, ref, grads
    for key, a in acc.items():
        assert a.error <= TOL, f"{key} all rows: {a.error:.3e}"


def test_radial_config5_full(cuda_device):
    from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct
    case = load_golden("full_radial_cfg5")
    c = R.CFG5
    d = R.cfg5_inputs()
    tp = UvuTensorProduct(c["u"], 1, c["m_max"], parity="full", parity_in2="canonical",
                          shared_weights=False)
    lin = torch.nn.Linear(c["hidden"], c["weight_numel"], bias=True)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(d["alpha"]))
        lin.bias.copy_(torch.from_numpy(d["bias"]))
    model = RadialUvuTensorProduct(tp, lin).to(cuda_device)
    nodes = torch.from_numpy(d["nodes"]).to(cuda_device)
    src = torch.from_numpy(d["src"]).to(cuda_device)
    x = nodes.index_select(0, src).requires_grad_(True)
    y = torch.from_numpy(d["angular"]).to(cuda_device).requires_grad_(True)
    h = torch.from_numpy(d["hidden"]).to(cuda_device).requires_grad_(True)
    g = torch.from_numpy(d["g"]).to(cuda_device)
    del d
    out = model(x, y, h)
    dx, dy, dh, da, db = torch.autograd.grad(
        out, (x, y, h, model.radial_out.weight, model.radial_out.bias), g)
    torch.cuda.synchronize()
    _check_rows_sums({"out": out.detach(), "dx": dx, "dy": dy, "dh": dh}, case,
                     case["keep_rows"])
    for key, value in (("da", da), ("db", db)):
        err = O.max_error(value.cpu().double().numpy(), case[f"{key}_f64"])
        assert err <= TOL, f"{key}: {err:.3e}"
