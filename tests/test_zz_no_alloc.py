"""ictc_o2_tp_backward_noalloc, the backward entry point for callers that cannot
allocate device memory (their allocator belongs to a host runtime or a pool they
must not bypass), called through the C-ABI and checked against
ictc_o2_tp_backward with a caller workspace.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import o2_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _inputs(rows, width, numel, seed, device):
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    x = torch.randn(rows, width, device=device, generator=gen)
    y = torch.randn(rows, width, device=device, generator=gen)
    g = torch.randn(rows, width, device=device, generator=gen)
    w = torch.randn(numel, device=device, generator=gen) * 0.1
    return x, y, w, g


def _backward_with_workspace(lib, x, y, w, g, channels, m_max, parity):
    from ictc_o2_hp_b200 import _lib
    rows = x.shape[0]
    need = _lib.tp_backward_workspace(rows, channels, m_max, "full" if parity else "canonical",
                                      x.device)
    workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=x.device)
    dx, dy, dw = torch.empty_like(x), torch.empty_like(y), torch.empty_like(w)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    status = lib.ictc_o2_tp_backward(x.data_ptr(), y.data_ptr(), w.data_ptr(), g.data_ptr(),
                                     dx.data_ptr(), dy.data_ptr(), dw.data_ptr(),
                                     workspace.data_ptr(), workspace.numel(), rows, channels,
                                     m_max, parity, 0, stream)
    assert status == 0, lib.ictc_o2_last_error().decode()
    return dx, dy, dw


def _backward_noalloc(lib, x, y, w, g, channels, m_max, parity):
    dx, dy, dw = torch.empty_like(x), torch.empty_like(y), torch.empty_like(w)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    status = lib.ictc_o2_tp_backward_noalloc(x.data_ptr(), y.data_ptr(), w.data_ptr(),
                                             g.data_ptr(), dx.data_ptr(), dy.data_ptr(),
                                             dw.data_ptr(), x.shape[0], channels, m_max, parity,
                                             0, stream)
    assert status == 0, lib.ictc_o2_last_error().decode()
    return dx, dy, dw


@pytest.mark.parametrize("channels,m_max,parity,rows", [
    (128, 6, 1, 4096),   # the benchmark configuration's shape
    (17, 3, 1, 301),     # ragged channel group
    (32, 2, 0, 1000),    # canonical parity
])
def test_noalloc_matches_workspace_entry_point(channels, m_max, parity, rows, cuda_device):
    from ictc_o2_hp_b200 import _lib
    lib = _lib.load()
    numel = _lib.tp_weight_numel(channels, m_max, "full" if parity else "canonical")
    width = O.TpOracle(channels, m_max, "full" if parity else "canonical").width
    # Two calls in a row with different inputs: the second must not see the
    # first call's scratch contents.
    for seed in (11, 12):
        x, y, w, g = _inputs(rows, width, numel, seed + channels, cuda_device)
        want = _backward_with_workspace(lib, x, y, w, g, channels, m_max, parity)
        got = _backward_noalloc(lib, x, y, w, g, channels, m_max, parity)
        torch.cuda.synchronize()
        for name, a, b in zip(("dx", "dy", "dw"), got, want):
            err = O.max_error(a.cpu().numpy(), b.cpu().numpy())
            assert err <= TOL, f"call {seed - 10} {name}: {err:.3e}"
    assert _lib.device_error() == 0


def test_noalloc_rejects_oversized_workspace(cuda_device):
    from ictc_o2_hp_b200 import _lib
    lib = _lib.load()
    # C = 32768 at m_max = 8: the prescaled weights and one partial weight-gradient
    # row alone exceed the fixed 32 MiB scratch; the call must fail before launching.
    channels, m_max = 32768, 8
    need = _lib.tp_backward_workspace(4096, channels, m_max, "full", cuda_device)
    assert need > 32 << 20
    status = lib.ictc_o2_tp_backward_noalloc(None, None, None, None, None, None, None, 4096,
                                             channels, m_max, 1, 0, None)
    assert status == _lib.ERR_WORKSPACE
    message = lib.ictc_o2_last_error().decode()
    assert "no-alloc" in message and "bytes of scratch" in message


def test_noalloc_zero_rows_zeroes_weight_gradient(cuda_device):
    from ictc_o2_hp_b200 import _lib
    lib = _lib.load()
    numel = _lib.tp_weight_numel(8, 2, "full")
    dw = torch.full((numel,), 7.0, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    status = lib.ictc_o2_tp_backward_noalloc(None, None, None, None, None, None, dw.data_ptr(),
                                             0, 8, 2, 1, 0, stream)
    assert status == 0, lib.ictc_o2_last_error().decode()
    torch.cuda.synchronize()
    assert np.all(dw.cpu().numpy() == 0.0)
