"""Row (edge) data parallelism across the GPUs of one node.

Every row of a tensor-product batch is independent; the only cross-row quantity is
the weight gradient (and, for the radial product, the affine-layer gradients).  So
each rank processes a contiguous shard of the rows with the single-GPU kernels and
the gradients of the module's parameters are summed with ONE all-reduce of one flat
buffer over NCCL (NVLink / NVSwitch).  No other exchange happens on the product
path.  For message passing over graphs whose nodes are partitioned over the ranks,
all_gather_rows / reduce_scatter_rows move node rows (the node-gradient
reduce-scatter is the adjoint of the node-feature all-gather).

The reference is single-GPU (it has no collective code); this module is the added
scaling layer.  Host logic is tested with the gloo backend on CPU.
"""

from __future__ import annotations

from datetime import timedelta
from typing import Iterable, Sequence

import torch
import torch.distributed as dist


def shard_bounds(rows: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous shard: equal shares, the remainder spread
    over the last ranks (one extra row each)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of {world}")
    if rows < 0:
        raise ValueError("rows must be >= 0")
    base, extra = divmod(rows, world)
    first_big = world - extra
    start = rank * base + max(0, rank - first_big)
    stop = start + base + (1 if rank >= first_big else 0)
    return start, stop


def shard_rows(tensor: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """Rank's slice of the leading (row) dimension."""
    start, stop = shard_bounds(tensor.shape[0], world, rank)
    return tensor[start:stop]


def allreduce_gradients(parameters: Iterable[torch.nn.Parameter],
                        group: dist.ProcessGroup | None = None,
                        average: bool = False) -> None:
    """Sums the gradients of `parameters` over the group with one collective on one
    flat buffer (parameters without a gradient contribute zeros)."""
    params = [p for p in parameters if p.requires_grad]
    if not params:
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    device = params[0].device
    dtype = params[0].dtype
    sizes = [p.numel() for p in params]
    flat = torch.empty(sum(sizes), device=device, dtype=dtype)
    offset = 0
    for p, n in zip(params, sizes):
        if p.grad is None:
            flat[offset:offset + n].zero_()
        else:
            flat[offset:offset + n].copy_(p.grad.reshape(-1))
        offset += n
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    if average:
        flat.div_(world)
    offset = 0
    for p, n in zip(params, sizes):
        view = flat[offset:offset + n].view_as(p)
        if p.grad is None:
            p.grad = view.clone()
        else:
            p.grad.copy_(view)
        offset += n


def init_process_group(backend: str | None = None, timeout_s: float = 120.0,
                       device: torch.device | None = None) -> tuple[int, int]:
    """Initialises the default group from the torchrun environment with a finite
    timeout, so a missing or failed rank ends collectives with an error instead of
    a hang.  Returns (rank, world)."""
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
    kwargs = {"timeout": timedelta(seconds=timeout_s)}
    if backend == "nccl" and device is not None:
        kwargs["device_id"] = device
    dist.init_process_group(backend, **kwargs)
    return dist.get_rank(), dist.get_world_size()


class RowParallel(torch.nn.Module):
    """Wraps a tensor-product module for row-sharded training: the caller passes the
    local shard of rows to forward(); after backward(), sync_gradients() sums the
    wrapped module's parameter gradients over the group (one all-reduce)."""

    def __init__(self, module: torch.nn.Module, group: dist.ProcessGroup | None = None):
        super().__init__()
        self.module = module
        self.group = group

    def forward(self, *args, **kwargs):
        return self.module(*args, **kwargs)

    def sync_gradients(self, average: bool = False) -> None:
        allreduce_gradients(self.module.parameters(), self.group, average)


# ------------------------------------------------------------ node-partitioned graphs
#
# For graphs whose nodes are partitioned over the ranks (rank r owns the contiguous
# node block shard_bounds(num_nodes, world, r)), a message-passing layer needs every
# node's features on the rank that holds an edge, and each node's summed messages
# (and each node's gradient) only on its owner:
#
#     h_all = all_gather_rows(h_own, counts)        # backward: node-gradient reduce-scatter
#     msg = graph.radial_messages(model, h_all, local_edges, angular, hidden)
#     partial = graph.scatter_sum(msg, local_edges) # this rank's edges' sums, every node
#     out_own = reduce_scatter_rows(partial, counts)  # backward: all-gather
#
# The two collectives are each other's adjoint, so autograd turns the forward
# all-gather of node features into a reduce-scatter of the node gradients: each rank
# receives the gradient of the nodes it owns, summed over every rank's edges, instead
# of an all-reduce of the whole node-gradient table.  Unequal blocks (the remainder on
# the last ranks) travel padded to the largest block.


def node_counts(num_nodes: int, world: int) -> list[int]:
    """Node-block sizes of the ranks (shard_bounds partition)."""
    return [b - a for a, b in (shard_bounds(num_nodes, world, r) for r in range(world))]


def _check_counts(counts: Sequence[int], group) -> int:
    world = dist.get_world_size(group)
    if len(counts) != world or any(int(c) < 0 for c in counts):
        raise ValueError(f"counts must hold {world} non-negative block sizes")
    return world


def _padded_all_gather(local: torch.Tensor, counts: Sequence[int], group) -> torch.Tensor:
    world = _check_counts(counts, group)
    rank = dist.get_rank(group)
    if local.shape[0] != counts[rank]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, counts say {counts[rank]}")
    biggest = max(counts)
    send = local.contiguous()
    if local.shape[0] != biggest:
        send = local.new_zeros((biggest, *local.shape[1:]))
        send[:local.shape[0]] = local
    recv = local.new_empty((world * biggest, *local.shape[1:]))
    dist.all_gather_into_tensor(recv, send, group=group)
    if all(c == biggest for c in counts):
        return recv
    return torch.cat([recv[r * biggest:r * biggest + n] for r, n in enumerate(counts)], dim=0)


def _padded_reduce_scatter(full: torch.Tensor, counts: Sequence[int], group) -> torch.Tensor:
    world = _check_counts(counts, group)
    rank = dist.get_rank(group)
    if full.shape[0] != sum(counts):
        raise ValueError(f"expected {sum(counts)} rows (all blocks), got {full.shape[0]}")
    biggest = max(counts)
    if all(c == biggest for c in counts):
        send = full.contiguous()
    else:
        send = full.new_zeros((world * biggest, *full.shape[1:]))
        start = 0
        for r, n in enumerate(counts):
            send[r * biggest:r * biggest + n] = full[start:start + n]
            start += n
    recv = full.new_empty((biggest, *full.shape[1:]))
    dist.reduce_scatter_tensor(recv, send, op=dist.ReduceOp.SUM, group=group)
    return recv[:counts[rank]]


class _AllGatherRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, local, counts, group):
        ctx.counts, ctx.group = counts, group
        return _padded_all_gather(local, counts, group)

    @staticmethod
    def backward(ctx, grad_full):
        return _padded_reduce_scatter(grad_full, ctx.counts, ctx.group), None, None


class _ReduceScatterRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, full, counts, group):
        ctx.counts, ctx.group = counts, group
        return _padded_reduce_scatter(full, counts, group)

    @staticmethod
    def backward(ctx, grad_local):
        return _padded_all_gather(grad_local, ctx.counts, ctx.group), None, None


def all_gather_rows(local: torch.Tensor, counts: Sequence[int],
                    group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """Every rank's row block, concatenated in rank order, on every rank.
    Differentiable: the gradient is the reduce-scatter of the incoming gradient, so
    each rank receives the sum over all ranks for the rows it owns."""
    counts = [int(c) for c in counts]
    return _AllGatherRows.apply(local, counts, group)


def reduce_scatter_rows(full: torch.Tensor, counts: Sequence[int],
                        group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """The rows of this rank's block, summed over every rank's `full` (one row per
    node of all blocks).  Differentiable: the gradient is the all-gather of the
    owners' gradients."""
    counts = [int(c) for c in counts]
    return _ReduceScatterRows.apply(full, counts, group)


def gather_rows(local: torch.Tensor, counts: Sequence[int],
                group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """Concatenates every rank's rows (shards of possibly unequal size) on all ranks;
    a convenience for checks and I/O, not used on the training path."""
    world = dist.get_world_size(group)
    width = local.shape[1:]
    biggest = max(counts)
    padded = local.new_zeros((biggest, *width))
    padded[:local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([part[:n] for part, n in zip(parts, counts)], dim=0)
