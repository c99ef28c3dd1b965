"""EdgeIndex validation (host logic, no GPU kernels)."""

from __future__ import annotations

import pytest
import torch


def test_edge_index_rejects_bad_inputs():
    from ictc_o2_hp_b200.graph import EdgeIndex
    with pytest.raises(ValueError, match="1-D int64"):
        EdgeIndex(torch.zeros(3, dtype=torch.int32), torch.zeros(3, dtype=torch.int64), 4)
    with pytest.raises(ValueError, match="CUDA"):
        EdgeIndex(torch.zeros(3, dtype=torch.int64), torch.zeros(3, dtype=torch.int64), 4)
    with pytest.raises(ValueError, match="1-D int64"):
        EdgeIndex(torch.zeros(2, 2, dtype=torch.int64), torch.zeros(4, dtype=torch.int64), 4)


def test_csr_groups_edges_stably():
    from ictc_o2_hp_b200.graph import _csr
    key = torch.tensor([2, 0, 2, 1, 0, 2])
    order, offsets = _csr(key, 4)
    assert order.tolist() == [1, 4, 3, 0, 2, 5]
    assert offsets.tolist() == [0, 2, 3, 6, 6]
