"""Node-partitioned message passing over NCCL on two GPUs: node features
all-gathered, messages gathered and summed by the graph kernels on each rank's edge
shard, node sums and node gradients reduce-scattered onto the owning ranks; checked
against the float64 single-process layer (gate 1e-5 normalised).  Needs two GPUs
(skipped otherwise, e.g. in the one-GPU suite)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import o2_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5
NODES, EDGES, WIDTH = 1001, 6000, 64


def _problem():
    gen = torch.Generator().manual_seed(11)
    h = torch.randn(NODES, WIDTH, generator=gen)
    src = torch.randint(0, NODES, (EDGES,), generator=gen)
    dst = torch.randint(0, NODES, (EDGES,), generator=gen)
    a = torch.randn(EDGES, WIDTH, generator=gen)
    cot = torch.randn(NODES, WIDTH, generator=gen)
    return h, src, dst, a, cot


def _worker(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    from ictc_o2_hp_b200.graph import EdgeIndex, gather, scatter_sum
    from ictc_o2_hp_b200.parallel import (all_gather_rows, node_counts, reduce_scatter_rows,
                                          shard_bounds)
    h, src, dst, a, cot = (t.to(device) for t in _problem())
    counts = node_counts(NODES, world)
    n0, n1 = shard_bounds(NODES, world, rank)
    e0, e1 = shard_bounds(EDGES, world, rank)
    edges = EdgeIndex(src[e0:e1].contiguous(), dst[e0:e1].contiguous(), NODES)
    h_own = h[n0:n1].clone().requires_grad_(True)
    h_all = all_gather_rows(h_own, counts)
    partial = scatter_sum(gather(h_all, edges) * a[e0:e1], edges)
    out_own = reduce_scatter_rows(partial, counts)
    (out_own * cot[n0:n1]).sum().backward()
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"out{rank}.npy"), out_own.detach().cpu().numpy())
    np.save(os.path.join(out_dir, f"dh{rank}.npy"), h_own.grad.cpu().numpy())
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


def test_node_partitioned_layer_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    h, src, dst, a, cot = (t.double() if t.is_floating_point() else t for t in _problem())
    hh = h.clone().requires_grad_(True)
    msg = hh.index_select(0, src) * a
    out = torch.zeros_like(h).index_add(0, dst, msg)
    (out * cot).sum().backward()
    from ictc_o2_hp_b200.parallel import shard_bounds
    for rank in range(2):
        n0, n1 = shard_bounds(NODES, 2, rank)
        got_out = np.load(tmp_path / f"out{rank}.npy")
        got_dh = np.load(tmp_path / f"dh{rank}.npy")
        assert O.max_error(got_out, out[n0:n1].detach().numpy()) <= TOL
        assert O.max_error(got_dh, hh.grad[n0:n1].numpy()) <= TOL
