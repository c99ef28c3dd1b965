"""TensorProductHostRunner: chunked, overlapped forward + VJP of host-resident rows
against the device path (the same kernels on device tensors): bit-identical out, dx
and dy; dw equal to the chunk-wise sum within the 1e-5 gate."""

from __future__ import annotations

import pytest
import torch

from oracle import o2_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("channels,m_max,parity,rows,chunk", [
    (16, 3, "full", 10000, 4096),   # three chunks, the last one ragged
    (32, 2, "canonical", 700, 4096),  # one partial chunk
    (8, 1, "full", 0, 128),         # no rows
    (128, 6, "full", 3000, 1024),   # the benchmark configuration's width
])
def test_runner_matches_device_path(channels, m_max, parity, rows, chunk, cuda_device):
    from ictc_o2_hp_b200 import TensorProduct
    from ictc_o2_hp_b200.host import TensorProductHostRunner
    torch.manual_seed(rows + channels)
    tp = TensorProduct(channels, m_max, parity=parity).to(cuda_device)
    W = tp.representation_dimension
    x, y, g = (torch.randn(rows, W).pin_memory() for _ in range(3))
    out, dx, dy = (torch.empty(rows, W).pin_memory() for _ in range(3))
    runner = TensorProductHostRunner(tp, chunk_rows=chunk)
    for _ in range(2):  # a second call reuses the buffers and events
        dw = runner.run(x, y, g, out, dx, dy)
        torch.cuda.current_stream().synchronize()
    xd, yd = x.to(cuda_device).requires_grad_(True), y.to(cuda_device).requires_grad_(True)
    ref = tp(xd, yd)
    rdx, rdy, rdw = torch.autograd.grad(ref, (xd, yd, tp.weight), g.to(cuda_device))
    assert torch.equal(out, ref.detach().cpu())
    assert torch.equal(dx, rdx.cpu()) and torch.equal(dy, rdy.cpu())
    if rows == 0:
        assert torch.count_nonzero(dw) == 0
    else:
        assert O.max_error(dw.cpu().numpy(), rdw.cpu().numpy()) <= 1e-5


def test_runner_rejects_device_or_misshaped_tensors(cuda_device):
    from ictc_o2_hp_b200 import TensorProduct
    from ictc_o2_hp_b200.host import TensorProductHostRunner
    tp = TensorProduct(8, 1).to(cuda_device)
    W = tp.representation_dimension
    runner = TensorProductHostRunner(tp)
    host = [torch.zeros(4, W) for _ in range(6)]
    with pytest.raises(ValueError, match="host float32"):
        runner.run(host[0].to(cuda_device), *host[1:])
    with pytest.raises(ValueError, match="same number of rows"):
        runner.run(host[0], host[1], host[2], torch.zeros(3, W), host[4], host[5])
