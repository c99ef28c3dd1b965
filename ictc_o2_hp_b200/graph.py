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
``torch.distributed.all_reduce``).  With the nodes partitioned over the ranks
instead, ``parallel.all_gather_rows`` brings every node's features to each rank and
``parallel.reduce_scatter_rows`` sums the partial node outputs onto their owners;
autograd turns the all-gather into the reduce-scatter of the node gradients.
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


# ------------------------------------------------- radial product over gathered rows


def _fused_gather() -> bool:
    """ICTC_RADIAL_GATHER=materialize gathers the rows into a copy first and runs the
    plain radial kernels (same results; for comparisons)."""
    import os
    return os.environ.get("ICTC_RADIAL_GATHER", "fused") != "materialize"


@torch.library.custom_op(f"{NAMESPACE}::radial_forward_gathered", mutates_args=())
def radial_forward_gathered(nodes: Tensor, index: Tensor, order: Tensor, offsets: Tensor,
                            angular: Tensor, hidden: Tensor, alpha: Tensor, bias: Tensor,
                            table: Tensor, rconfig: list[int], has_bias: bool) -> Tensor:
    """uvu(nodes[index], angular, hidden @ alpha^T + bias): the radial product with
    the node gather folded into the edge kernels (ictc_o2_radial_forward_gathered);
    order / offsets (the CSR of index) serve the adjoint.  Configurations the edge
    tile does not cover gather the rows first."""
    from .ops import require_cuda_float32
    require_cuda_float32("radial messages", nodes, angular, hidden, alpha)
    nodes, angular, hidden = nodes.contiguous(), angular.contiguous(), hidden.contiguous()
    alpha = alpha.contiguous()
    bias_c = bias.contiguous() if has_bias else None
    out = nodes.new_empty(index.shape[0], nodes.shape[1])
    with torch.cuda.device(nodes.device):
        fwd, _ = _lib.radial_workspace(rconfig, index.shape[0], nodes.device)
        workspace = torch.empty(max(fwd, 16), dtype=torch.uint8, device=nodes.device)
        try:
            if not _fused_gather():
                raise NotImplementedError
            _lib.radial_forward_gathered(nodes, index, angular, hidden, alpha, bias_c, out,
                                         rconfig, table, workspace)
        except NotImplementedError:
            left = nodes.index_select(0, index)
            _lib.radial_forward(left, angular, hidden, alpha, bias_c, out, rconfig, table,
                                workspace)
    return out


@radial_forward_gathered.register_fake
def _radial_forward_gathered_fake(nodes, index, order, offsets, angular, hidden, alpha, bias,
                                  table, rconfig, has_bias):
    return nodes.new_empty(index.shape[0], nodes.shape[1])


@torch.library.custom_op(f"{NAMESPACE}::radial_backward_gathered", mutates_args=())
def radial_backward_gathered(nodes: Tensor, index: Tensor, angular: Tensor, hidden: Tensor,
                             alpha: Tensor, bias: Tensor, grad_output: Tensor, table: Tensor,
                             rconfig: list[int], has_bias: bool, needed: int
                             ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """(per-edge gradient of the gathered rows, g_angular, g_hidden, g_alpha, g_bias)
    for the role mask `needed` (1, 2, 4, 8, 16); absent roles are empty."""
    from .ops import require_cuda_float32
    require_cuda_float32("radial messages backward", nodes, angular, hidden, alpha, grad_output)
    nodes, angular, hidden = nodes.contiguous(), angular.contiguous(), hidden.contiguous()
    alpha, grad_output = alpha.contiguous(), grad_output.contiguous()
    if not has_bias:
        needed &= ~16
    bias_c = bias.contiguous() if has_bias else None
    rows = index.shape[0]
    want_xy = bool(needed & 3)
    gx = nodes.new_empty(rows, nodes.shape[1]) if want_xy else nodes.new_empty(0)
    gy = torch.empty_like(angular) if want_xy else angular.new_empty(0)
    gh = torch.empty_like(hidden) if needed & 4 else hidden.new_empty(0)
    ga = torch.empty_like(alpha) if needed & 24 else alpha.new_empty(0)
    gb = torch.empty_like(bias) if needed & 16 else alpha.new_empty(0)
    mask = needed | (3 if want_xy else 0) | (8 if needed & 16 else 0)
    args = (gx if want_xy else None, gy if want_xy else None, gh if needed & 4 else None,
            ga if needed & 24 else None, gb if needed & 16 else None)
    with torch.cuda.device(nodes.device):
        _, bwd = _lib.radial_workspace(rconfig, rows, nodes.device)
        workspace = torch.empty(max(bwd, 16), dtype=torch.uint8, device=nodes.device)
        try:
            if not _fused_gather():
                raise NotImplementedError
            _lib.radial_backward_gathered(nodes, index, angular, hidden, alpha, bias_c,
                                          grad_output, *args, rconfig, mask, table, workspace)
        except NotImplementedError:
            left = nodes.index_select(0, index)
            _lib.radial_backward(left, angular, hidden, alpha, bias_c, grad_output, *args,
                                 rconfig, mask, table, workspace)
    return (gx if needed & 1 else nodes.new_empty(0), gy if needed & 2 else angular.new_empty(0),
            gh, ga if needed & 8 else alpha.new_empty(0), gb)


@radial_backward_gathered.register_fake
def _radial_backward_gathered_fake(nodes, index, angular, hidden, alpha, bias, grad_output, table,
                                   rconfig, has_bias, needed):
    if not has_bias:
        needed &= ~16
    rows = index.shape[0]
    return (nodes.new_empty(rows, nodes.shape[1]) if needed & 1 else nodes.new_empty(0),
            torch.empty_like(angular) if needed & 2 else angular.new_empty(0),
            torch.empty_like(hidden) if needed & 4 else hidden.new_empty(0),
            torch.empty_like(alpha) if needed & 8 else alpha.new_empty(0),
            torch.empty_like(bias) if needed & 16 else alpha.new_empty(0))


def _gathered_setup(ctx, inputs, output):
    nodes, index, order, offsets, angular, hidden, alpha, bias, table, rconfig, has_bias = inputs
    ctx.save_for_backward(nodes, index, order, offsets, angular, hidden, alpha, bias, table)
    ctx.rconfig, ctx.has_bias = rconfig, has_bias


def _gathered_autograd(ctx, grad_output):
    if torch.is_grad_enabled():
        raise NotImplementedError(
            "second derivatives through radial_messages are not available; use "
            "gather(nodes, edges) and the RadialUvuTensorProduct module for them")
    nodes, index, order, offsets, angular, hidden, alpha, bias, table = ctx.saved_tensors
    need = ctx.needs_input_grad
    flags = [need[0], need[4], need[5], need[6], need[7] and ctx.has_bias]
    needed = sum(int(f) << i for i, f in enumerate(flags))
    if needed == 0:
        return (None,) * 11
    gx, gy, gh, ga, gb = radial_backward_gathered(nodes, index, angular, hidden, alpha, bias,
                                                  grad_output.contiguous(), table, ctx.rconfig,
                                                  ctx.has_bias, needed)
    g_nodes = segment_sum(gx, index, order, offsets) if flags[0] else None
    return (g_nodes, None, None, None, gy if flags[1] else None, gh if flags[2] else None,
            ga if flags[3] else None, gb if flags[4] else None, None, None, None)


radial_forward_gathered.register_autograd(_gathered_autograd, setup_context=_gathered_setup)


def radial_messages(model, nodes: Tensor, edges: EdgeIndex, angular: Tensor,
                    radial_hidden: Tensor, which: str = "src") -> Tensor:
    """Per-edge messages ``model(gather(nodes, edges, which), angular, radial_hidden)``
    of a RadialUvuTensorProduct ``model``, with the gather folded into the radial
    kernels: the [num_edges, width1] gathered copy of the node features is never
    written.  The node-feature gradient sums the per-edge gradients in the edges'
    CSR order (deterministic), as the adjoint of ``gather`` does, so the result is
    the same as that of ``model(gather(nodes, edges, which), ...)``, bit for bit.
    Second derivatives are not available through this fused form; use ``gather``
    and the module for them."""
    tp = model.tp
    if nodes.dim() != 2 or nodes.shape[1] != tp.input1_dimension:
        raise ValueError("nodes must be [num_nodes, tp.input1_dimension]")
    if nodes.shape[0] != edges.num_nodes:
        raise ValueError("nodes must have one row per node of the EdgeIndex")
    E = edges.num_edges
    if angular.shape != (E, tp.input2_dimension):
        raise ValueError("angular must be [num_edges, tp.input2_dimension]")
    if radial_hidden.shape != (E, model.radial_out.in_features):
        raise ValueError("radial_hidden must be [num_edges, radial_out.in_features]")
    index, order, offsets = edges.csr(which)
    bias = model.radial_out.bias
    has_bias = bias is not None
    return radial_forward_gathered(nodes, index, order, offsets, angular, radial_hidden,
                                   model.radial_out.weight,
                                   bias if has_bias else model.radial_out.weight.new_empty(0),
                                   tp._table, model._rconfig(), has_bias)
