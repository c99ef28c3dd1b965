"""Message passing around the radial product: node gather and message sum.

A layer gathers node features to its edges (``x_e = nodes[src_e]``), runs the edge
product, and sums the messages into the destination nodes (``out_n = sum of
messages with dst_e = n``).  The reference stops at the edge product
(docs/RADIAL.md:97-99); these two steps are the kernels ``ictc_o2_gather_rows`` and
``ictc_o2_segment_sum``, each the other's adjoint, with the summation order fixed
by a stable sort of the edges, so node outputs and node gradients are bit-identical
from run to run (no atomics).

    edges = EdgeIndex(src, dst, num_nodes)          # once per graph
    x = gather(nodes, edges)                        # [E, W] from [num_nodes, W]
    out = scatter_sum(messages, edges)              # [num_nodes, W] from [E, W]

Edge-sharded data parallelism: each rank builds the EdgeIndex of its edge shard
against the full node set; the per-rank node sums are partial and add up with one
all-reduce (``ictc_o2_hp_b200.parallel.allreduce_gradients`` or
``torch.distributed.all_reduce``).
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib
from .ops import NAMESPACE


def _csr(key: Tensor, num_nodes: int) -> tuple[Tensor, Tensor]:
    """Edges grouped by `key` (a stable sort: equal keys keep edge order) and the
    groups' CSR pointers [num_nodes + 1]."""
    order = torch.sort(key, stable=True).indices
    counts = torch.bincount(key, minlength=num_nodes)
    offsets = torch.zeros(num_nodes + 1, dtype=torch.int64, device=key.device)
    torch.cumsum(counts, 0, out=offsets[1:])
    return order, offsets


class EdgeIndex:
    """Source and destination of every edge (int64, on the GPU) and the CSR orders
    of both, built once per graph."""

    def __init__(self, src: Tensor, dst: Tensor, num_nodes: int):
        for name, t in (("src", src), ("dst", dst)):
            if t.dim() != 1 or t.dtype != torch.int64:
                raise ValueError(f"{name} must be a 1-D int64 tensor")
            if t.device.type != "cuda":
                raise ValueError(f"{name} must be on a CUDA device")
        if src.shape != dst.shape or src.device != dst.device:
            raise ValueError("src and dst must have the same length and device")
        if int(num_nodes) < 0:
            raise ValueError("num_nodes must be >= 0")
        self.num_nodes = int(num_nodes)
        self.src, self.dst = src.contiguous(), dst.contiguous()
        if self.src.numel():
            lo = torch.minimum(self.src.min(), self.dst.min())
            hi = torch.maximum(self.src.max(), self.dst.max())
            if int(lo) < 0 or int(hi) >= self.num_nodes:
                raise ValueError("edge endpoints must lie in [0, num_nodes)")
        self._by = {"src": _csr(self.src, self.num_nodes), "dst": _csr(self.dst, self.num_nodes)}

    @property
    def num_edges(self) -> int:
        return self.src.numel()

    def csr(self, which: str) -> tuple[Tensor, Tensor, Tensor]:
        """(index, order, offsets) of the edges grouped by `which` ("src" or "dst")."""
        if which not in self._by:
            raise ValueError("which must be 'src' or 'dst'")
        return (self.src if which == "src" else self.dst, *self._by[which])


def _check_rows(name: str, t: Tensor) -> None:
    if t.device.type != "cuda" or t.dtype != torch.float32 or t.dim() != 2:
        raise ValueError(f"{name} must be a 2-D float32 CUDA tensor")


@torch.library.custom_op(f"{NAMESPACE}::gather_rows", mutates_args=())
def gather_rows(source: Tensor, index: Tensor, order: Tensor, offsets: Tensor) -> Tensor:
    """out[e] = source[index[e]] (order / offsets: the CSR of index, for the adjoint)."""
    _check_rows("source", source)
    source = source.contiguous()
    out = torch.empty(index.shape[0], source.shape[1], dtype=source.dtype, device=source.device)
    with torch.cuda.device(source.device):
        _lib.gather_rows(source, index, out)
    return out


@gather_rows.register_fake
def _gather_rows_fake(source, index, order, offsets):
    return source.new_empty(index.shape[0], source.shape[1])


@torch.library.custom_op(f"{NAMESPACE}::segment_sum", mutates_args=())
def segment_sum(values: Tensor, index: Tensor, order: Tensor, offsets: Tensor) -> Tensor:
    """out[n] = sum of values[e] with index[e] = n, in the fixed order `order`."""
    _check_rows("values", values)
    values = values.contiguous()
    out = torch.empty(offsets.shape[0] - 1, values.shape[1], dtype=values.dtype,
                      device=values.device)
    with torch.cuda.device(values.device):
        _lib.segment_sum(values, offsets, order, out)
    return out


@segment_sum.register_fake
def _segment_sum_fake(values, index, order, offsets):
    return values.new_empty(offsets.shape[0] - 1, values.shape[1])


def _graph_setup(ctx, inputs, output):
    _, index, order, offsets = inputs
    ctx.save_for_backward(index, order, offsets)


def _gather_backward(ctx, grad):
    index, order, offsets = ctx.saved_tensors
    return segment_sum(grad.contiguous(), index, order, offsets), None, None, None


def _segment_sum_backward(ctx, grad):
    index, order, offsets = ctx.saved_tensors
    return gather_rows(grad.contiguous(), index, order, offsets), None, None, None


gather_rows.register_autograd(_gather_backward, setup_context=_graph_setup)
segment_sum.register_autograd(_segment_sum_backward, setup_context=_graph_setup)


def gather(nodes: Tensor, edges: EdgeIndex, which: str = "src") -> Tensor:
    """Node features of each edge's `which` endpoint: [num_edges, W]."""
    if nodes.shape[0] != edges.num_nodes:
        raise ValueError("nodes must have one row per node of the EdgeIndex")
    return gather_rows(nodes, *edges.csr(which))


def scatter_sum(messages: Tensor, edges: EdgeIndex, which: str = "dst") -> Tensor:
    """Sum of each node's incoming (`which` = "dst") edge messages: [num_nodes, W]."""
    if messages.shape[0] != edges.num_edges:
        raise ValueError("messages must have one row per edge of the EdgeIndex")
    return segment_sum(messages, *edges.csr(which))
