"""GPU parity of the fused radial kernels (through the C-ABI) against the reference's
golden fixtures and the CPU oracle; gate 1e-5 normalised max error."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import o2_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def build(u, m_max, hidden, bias, device, alpha=None, b=None):
    from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct
    tp = UvuTensorProduct(u, 1, m_max, parity="full", parity_in2="canonical",
                          shared_weights=False)
    lin = torch.nn.Linear(hidden, tp.weight_numel, bias=bias)
    with torch.no_grad():
        if alpha is not None:
            lin.weight.copy_(torch.as_tensor(alpha))
        if bias and b is not None:
            lin.bias.copy_(torch.as_tensor(b))
    return RadialUvuTensorProduct(tp, lin).to(device)


def run(module, x, y, h, g, device):
    xx, yy, hh = (torch.as_tensor(a, dtype=torch.float32, device=device).requires_grad_(True)
                  for a in (x, y, h))
    out = module(xx, yy, hh)
    params = [module.radial_out.weight] + (
        [module.radial_out.bias] if module.radial_out.bias is not None else [])
    grads = torch.autograd.grad(out, (xx, yy, hh, *params), torch.as_tensor(g, device=device))
    torch.cuda.synchronize()
    return [out.detach().cpu().numpy()] + [t.cpu().numpy() for t in grads]


@pytest.mark.parametrize("name", golden_names("radial_"))
def test_golden(name, cuda_device):
    c = load_golden(name)
    bias = bool(c["bias"])
    module = build(int(c["u"]), int(c["m_max"]), int(c["hidden"]), bias, cuda_device,
                   c["alpha"], c["b"] if bias else None)
    got = run(module, c["x"], c["y"], c["h"], c["g"], cuda_device)
    keys = ["out", "dx", "dy", "dh", "da"] + (["db"] if bias else [])
    for key, value in zip(keys, got):
        err = O.max_error(value, c[f"{key}_f64"])
        assert err <= TOL, f"{key}: {err:.3e}"


@pytest.mark.parametrize("u,m_max,hidden,bias,rows", [
    (64, 3, 64, False, 300),   # benchmark config 5 shape
    (64, 3, 64, True, 97),
    (17, 2, 9, True, 70),
    (128, 1, 40, False, 33),
    (3, 0, 5, True, 11),
    (16, 5, 12, True, 45),     # second input wider than 8 values
    (72, 2, 64, False, 130),   # two channel tiles in the weight gradient
    (32, 2, 512, True, 150),   # hidden too wide to stay resident: row-tile fallback
    (160, 2, 24, True, 70),    # two channel tiles, the last one partial
    (256, 1, 16, False, 50),   # two full channel tiles
])
def test_against_oracle(u, m_max, hidden, bias, rows, cuda_device):
    oracle_tp = O.UvuOracle(u, 1, m_max, "full", "canonical")
    radial = O.RadialOracle(oracle_tp)
    rng = np.random.default_rng(u + 7 * hidden + rows)
    Wn = oracle_tp.weight_numel
    alpha = (rng.standard_normal((Wn, hidden)) / np.sqrt(hidden)).astype(np.float32)
    b = rng.standard_normal(Wn).astype(np.float32) if bias else None
    x = rng.standard_normal((rows, oracle_tp.width1)).astype(np.float32)
    theta = rng.uniform(0, 2 * np.pi, rows)
    y = np.concatenate([np.ones((rows, 1))] + [
        np.stack([np.cos(m * theta), np.sin(m * theta)], -1) for m in range(1, m_max + 1)],
        axis=-1).astype(np.float32)
    h = rng.standard_normal((rows, hidden)).astype(np.float32)
    g = rng.standard_normal((rows, oracle_tp.width1)).astype(np.float32)
    want = radial.vjp(*(a.astype(np.float64) for a in (x, y, h, alpha, g)),
                      bias=None if b is None else b.astype(np.float64))
    module = build(u, m_max, hidden, bias, cuda_device, alpha, b)
    got = run(module, x, y, h, g, cuda_device)
    keys = ["out", "dx", "dy", "dh", "da"] + (["db"] if bias else [])
    for key, a, w in zip(keys, got, want):
        err = O.max_error(a, w)
        assert err <= TOL, f"{key}: {err:.3e}"


@pytest.mark.parametrize("shape", ["split", "wide", "mid"])
@pytest.mark.parametrize("u,m_max,hidden,bias,rows", [
    (64, 3, 64, True, 300),    # channel tile of 64
    (160, 2, 24, True, 70),    # channel tiles of 128, the last partial
])
def test_thread_tile_shapes(shape, u, m_max, hidden, bias, rows, cuda_device, monkeypatch):
    """Every edge-tile shape for both the forward and the dx tile
    (ICTC_RADIAL_TILE=split: 4 x 8 on 256 threads, wide: 4 x 4 on 512, mid: 4 x 4 on 384)
    against the oracle; the defaults (wide forward, mid dx tile) run every other case."""
    monkeypatch.setenv("ICTC_RADIAL_TILE", shape)
    test_against_oracle(u, m_max, hidden, bias, rows, cuda_device)


def test_role_pruning_matches_full(cuda_device):
    """Requesting a subset of gradients returns the same values as the full VJP."""
    torch.manual_seed(0)
    module = build(16, 2, 8, True, cuda_device)
    tp = module.tp
    x = torch.randn(50, tp.input1_dimension, device=cuda_device, requires_grad=True)
    y = torch.randn(50, tp.input2_dimension, device=cuda_device, requires_grad=True)
    h = torch.randn(50, 8, device=cuda_device, requires_grad=True)
    full = torch.autograd.grad(module(x, y, h).square().sum(),
                               (x, y, h, module.radial_out.weight, module.radial_out.bias))
    only_bias = torch.autograd.grad(module(x, y, h).square().sum(), (module.radial_out.bias,))
    only_h = torch.autograd.grad(module(x, y, h).square().sum(), (h,))
    assert torch.equal(only_bias[0], full[4]) and torch.equal(only_h[0], full[2])


def test_compile_and_validation(cuda_device):
    from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct
    torch.manual_seed(1)
    module = build(8, 2, 6, True, cuda_device)
    tp = module.tp
    x = torch.randn(40, tp.input1_dimension, device=cuda_device)
    y = torch.randn(40, tp.input2_dimension, device=cuda_device)
    h = torch.randn(40, 6, device=cuda_device)
    compiled = torch.compile(module, fullgraph=True, dynamic=False)
    assert torch.equal(compiled(x, y, h), module(x, y, h))
    with pytest.raises(ValueError):
        RadialUvuTensorProduct(UvuTensorProduct(4, 2, 1, shared_weights=False),
                               torch.nn.Linear(3, 10))
    with pytest.raises(ValueError):
        module(x, y[:, :-1], h)
