"""Device-side error reporting of the bounded waits.  Every staged kernel waits on
mbarriers with a time limit (2 s of the GPU's global timer); when it runs out the
kernel records a code in its unit's device error flag and exits, and
ictc_o2_device_error() reads and clears the flags of every unit.  The probe test
makes one such wait run out on purpose, on a barrier that nothing arrives at, with
no copy in flight; the others check that no product leaves a code behind."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_probe_runs_out_and_reports(cuda_device):
    from ictc_o2_hp_b200 import _lib
    assert _lib.device_error() == 0
    waited = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    _lib.test_wait_timeout(1000, waited)       # 1 ms limit
    assert _lib.device_error() == 13           # synchronizes, reads and clears
    assert int(waited.item()) == 0
    assert _lib.device_error() == 0
    # the context stays usable
    x = torch.ones(4, device=cuda_device)
    assert float((x * 2).sum()) == 8.0


def test_no_code_left_by_any_product(cuda_device):
    """Shared-weight uvu, per-row uvu (quad and streamed kernels) and the radial
    tile each run their staged loops; every unit's flag stays clear."""
    from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct, _lib
    assert _lib.device_error() == 0
    torch.manual_seed(0)
    shared = UvuTensorProduct(64, 8, 2).to(cuda_device)
    x = torch.randn(300, shared.input1_dimension, device=cuda_device, requires_grad=True)
    y = torch.randn(300, shared.input2_dimension, device=cuda_device, requires_grad=True)
    torch.autograd.grad(shared(x, y).sum(), (x, y, shared.weight))
    per_row = UvuTensorProduct(64, 8, 2, shared_weights=False).to(cuda_device)
    w = torch.randn(300, per_row.weight_numel, device=cuda_device, requires_grad=True)
    torch.autograd.grad(per_row(x, y, w).sum(), (x, y, w))
    tp = UvuTensorProduct(64, 1, 3, parity="full", parity_in2="canonical",
                          shared_weights=False)
    radial = RadialUvuTensorProduct(tp, torch.nn.Linear(16, tp.weight_numel)).to(cuda_device)
    xr = torch.randn(500, tp.input1_dimension, device=cuda_device, requires_grad=True)
    yr = torch.randn(500, tp.input2_dimension, device=cuda_device, requires_grad=True)
    hr = torch.randn(500, 16, device=cuda_device, requires_grad=True)
    torch.autograd.grad(radial(xr, yr, hr).sum(), (xr, yr, hr, radial.radial_out.weight))
    assert _lib.device_error() == 0
