"""Row sharding and the single gradient all-reduce, on CPU with gloo ranks
(world_size 2), including a rank that fails before the collective."""

from __future__ import annotations

import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ictc_o2_hp_b200.parallel import (all_gather_rows, allreduce_gradients, node_counts,
                                      reduce_scatter_rows, shard_bounds, shard_rows)


@pytest.mark.parametrize("rows", [0, 1, 5, 64, 65537])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_bounds_partition(rows, world):
    bounds = [shard_bounds(rows, world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == rows
    for (a, b), (c, d) in zip(bounds, bounds[1:]):
        assert b == c
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes)  # the remainder sits on the last ranks


def test_shard_bounds_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)
    with pytest.raises(ValueError):
        shard_bounds(-1, 2, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    from ictc_o2_hp_b200.ops import tp_plan, torch_tp_flat
    plan = tp_plan(8, 3, "full", "component")
    torch.manual_seed(0)
    rows = 37
    x = torch.randn(rows, plan.representation_dimension, dtype=torch.float64)
    y = torch.randn_like(x)
    g = torch.randn_like(x)
    w = torch.nn.Parameter(torch.randn(plan.weight_numel, dtype=torch.float64))
    xs, ys, gs = (shard_rows(t, world, rank) for t in (x, y, g))
    out = torch_tp_flat(xs, ys, w, plan)
    out.backward(gs)
    allreduce_gradients([w])
    np.save(os.path.join(result_dir, f"dw{rank}.npy"), w.grad.numpy())
    dist.destroy_process_group()


def test_sharded_weight_gradient_equals_full_batch(tmp_path):
    """Two gloo ranks each take a row shard; after one all-reduce the weight
    gradient equals the full-batch gradient on both ranks."""
    port = _free_port()
    mp.spawn(_tp_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    from ictc_o2_hp_b200.ops import tp_plan, torch_tp_flat
    plan = tp_plan(8, 3, "full", "component")
    torch.manual_seed(0)
    x = torch.randn(37, plan.representation_dimension, dtype=torch.float64)
    y = torch.randn_like(x)
    g = torch.randn_like(x)
    w = torch.nn.Parameter(torch.randn(plan.weight_numel, dtype=torch.float64))
    torch_tp_flat(x, y, w, plan).backward(g)
    for rank in range(2):
        got = np.load(tmp_path / f"dw{rank}.npy")
        assert np.abs(got - w.grad.numpy()).max() < 1e-12


def _failing_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        # this rank dies between steps, before the collective
        os._exit(0)
    w = torch.nn.Parameter(torch.ones(4))
    w.grad = torch.ones(4)
    start = time.monotonic()
    status = "no error"
    try:
        allreduce_gradients([w])
    except Exception as exc:  # a finite-timeout group reports the missing peer
        status = f"error: {type(exc).__name__}"
    with open(os.path.join(result_dir, "rank0.txt"), "w") as fh:
        fh.write(f"{status}\n{time.monotonic() - start:.1f}\n")
    os._exit(0)


def test_missing_rank_ends_collective_with_error(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung past the process-group timeout")
    status, elapsed = (tmp_path / "rank0.txt").read_text().splitlines()[:2]
    assert status.startswith("error"), status
    assert float(elapsed) < 90


def _graph_problem():
    """A small graph (float64): node features, per-edge factors, a node cotangent."""
    gen = torch.Generator().manual_seed(7)
    nodes, edges, width = 11, 40, 5
    h = torch.randn(nodes, width, dtype=torch.float64, generator=gen)
    src = torch.randint(0, nodes, (edges,), generator=gen)
    dst = torch.randint(0, nodes, (edges,), generator=gen)
    a = torch.randn(edges, width, dtype=torch.float64, generator=gen)
    cot = torch.randn(nodes, width, dtype=torch.float64, generator=gen)
    return h, src, dst, a, cot


def _layer(h_all, src, dst, a, nodes):
    """Messages h[src] * a summed into the destinations (index_select / index_add_
    stand in for the gather and segment-sum kernels on the CPU)."""
    msg = h_all.index_select(0, src) * a
    return torch.zeros(nodes, h_all.shape[1], dtype=h_all.dtype).index_add(0, dst, msg)


def _node_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    h, src, dst, a, cot = _graph_problem()
    counts = node_counts(h.shape[0], world)
    n0, n1 = shard_bounds(h.shape[0], world, rank)
    e0, e1 = shard_bounds(src.shape[0], world, rank)
    h_own = h[n0:n1].clone().requires_grad_(True)
    h_all = all_gather_rows(h_own, counts)
    partial = _layer(h_all, src[e0:e1], dst[e0:e1], a[e0:e1], h.shape[0])
    out_own = reduce_scatter_rows(partial, counts)
    (out_own * cot[n0:n1]).sum().backward()
    np.save(os.path.join(result_dir, f"out{rank}.npy"), out_own.detach().numpy())
    np.save(os.path.join(result_dir, f"dh{rank}.npy"), h_own.grad.numpy())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_node_partitioned_message_passing(tmp_path, world):
    """Nodes split over gloo ranks (11 nodes: unequal blocks), edges sharded: the
    all-gather of node features and the reduce-scatter of the message sums give each
    rank its own nodes' outputs, and autograd's reduce-scatter of the node gradients
    gives each rank its own nodes' gradients, equal to the single-process layer."""
    port = _free_port()
    mp.spawn(_node_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    h, src, dst, a, cot = _graph_problem()
    hh = h.clone().requires_grad_(True)
    out = _layer(hh, src, dst, a, h.shape[0])
    (out * cot).sum().backward()
    for rank in range(world):
        n0, n1 = shard_bounds(h.shape[0], world, rank)
        got_out = np.load(tmp_path / f"out{rank}.npy")
        got_dh = np.load(tmp_path / f"dh{rank}.npy")
        assert np.abs(got_out - out[n0:n1].detach().numpy()).max() < 1e-12
        assert np.abs(got_dh - hh.grad[n0:n1].numpy()).max() < 1e-12
