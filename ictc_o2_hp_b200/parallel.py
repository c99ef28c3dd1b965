"""Row (edge) data parallelism across the GPUs of one node.

Every row of a tensor-product batch is independent; the only cross-row quantity is
the weight gradient (and, for the radial product, the affine-layer gradients).  So
each rank processes a contiguous shard of the rows with the single-GPU kernels and
the gradients of the module's parameters are summed with ONE all-reduce of one flat
buffer over NCCL (NVLink / NVSwitch).  No other exchange happens.

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
