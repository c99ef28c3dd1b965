"""torch.library custom ops over the C-ABI kernels, with fake (meta) kernels for
torch.compile and autograd formulas.

Replaces the reference's ``o2_forward`` / ``o2_backward`` Triton ops
(src/ictc_o2_hp/triton_o2.py:786-966, autograd :1035-1092).  The path metadata
tensors and global metadata registry of the reference become plain integer and
string arguments.  Inputs must be CUDA float32: there is no CPU fallback.
Second derivatives recompute a differentiable PyTorch formula on the GPU, as
the reference does (triton_o2.py:969-1069).
"""

from __future__ import annotations

from functools import lru_cache

import torch
from torch import Tensor

from . import _lib
from ._algebra import MAGNITUDES, TpPlan

NAMESPACE = "ictc_o2_b200"


def require_cuda_float32(what: str, *tensors: Tensor) -> None:
    device = tensors[0].device
    for t in tensors:
        if t.device.type != "cuda" or t.dtype != torch.float32:
            raise TypeError(
                f"{what} runs only on CUDA float32 tensors (this implementation has no CPU "
                f"or other-dtype fallback); got {t.dtype} on {t.device}")
        if t.device != device:
            raise ValueError(f"{what}: all operands must be on one device")


@lru_cache(maxsize=None)
def tp_plan(channels: int, m_max: int, parity: str, normalization: str) -> TpPlan:
    return TpPlan(channels, m_max, parity, normalization)


# ----------------------------------------------------------------- TensorProduct


@torch.library.custom_op(f"{NAMESPACE}::tp_forward", mutates_args=())
def tp_forward(left: Tensor, right: Tensor, weight: Tensor, channels: int, m_max: int,
               parity: str, normalization: str) -> Tensor:
    """out[N, W] of TensorProduct on flat rows (triton_o2.py:786-875)."""
    require_cuda_float32("TensorProduct", left, right, weight)
    left, right, weight = left.contiguous(), right.contiguous(), weight.contiguous()
    out = torch.empty_like(left)
    with torch.cuda.device(left.device):
        _lib.tp_forward(left, right, weight, out, channels, m_max, parity, normalization)
    return out


@tp_forward.register_fake
def _tp_forward_fake(left, right, weight, channels, m_max, parity, normalization):
    return torch.empty_like(left)


@torch.library.custom_op(f"{NAMESPACE}::tp_backward", mutates_args=())
def tp_backward(left: Tensor, right: Tensor, weight: Tensor, grad_output: Tensor, channels: int,
                m_max: int, parity: str, normalization: str) -> tuple[Tensor, Tensor, Tensor]:
    """(dx, dy, dw) of TensorProduct (triton_o2.py:878-966)."""
    require_cuda_float32("TensorProduct backward", left, right, weight, grad_output)
    left, right = left.contiguous(), right.contiguous()
    weight, grad_output = weight.contiguous(), grad_output.contiguous()
    grad_left, grad_right = torch.empty_like(left), torch.empty_like(right)
    grad_weight = torch.empty_like(weight)
    with torch.cuda.device(left.device):
        size = _lib.tp_backward_workspace(left.shape[0], channels, m_max, parity, left.device)
        workspace = torch.empty(max(size, 1), dtype=torch.uint8, device=left.device)
        _lib.tp_backward(left, right, weight, grad_output, grad_left, grad_right, grad_weight,
                         workspace, channels, m_max, parity, normalization)
    return grad_left, grad_right, grad_weight


@tp_backward.register_fake
def _tp_backward_fake(left, right, weight, grad_output, channels, m_max, parity, normalization):
    return torch.empty_like(left), torch.empty_like(right), torch.empty_like(weight)


def _tp_setup(ctx, inputs, output):
    left, right, weight, channels, m_max, parity, normalization = inputs
    ctx.save_for_backward(left, right, weight)
    ctx.config = (channels, m_max, parity, normalization)


def _tp_autograd(ctx, grad_output):
    left, right, weight = ctx.saved_tensors
    gx, gy, gw = tp_backward(left, right, weight, grad_output.contiguous(), *ctx.config)
    return gx, gy, gw, None, None, None, None


tp_forward.register_autograd(_tp_autograd, setup_context=_tp_setup)


def torch_tp_flat(left: Tensor, right: Tensor, weight: Tensor, plan: TpPlan) -> Tensor:
    """Differentiable PyTorch formula of the same map, used for second derivatives
    only (the role of triton_o2.py:969-1032)."""
    n, C = left.shape[0], plan.channels
    offsets = plan.key_offsets()
    mags = MAGNITUDES[plan.normalization]

    def split(value):
        blocks = {}
        for b in plan.blocks:
            o = offsets[b.key]
            v = value[:, o:o + b.multiplicity * b.irrep_dimension].reshape(
                n, b.parity_copies, C, b.irrep_dimension)
            if b.parity_copies == 2:
                v = torch.cat((v[:, :1], torch.stack((-v[:, 1, :, 1], v[:, 1, :, 0]), -1)[:, None]),
                              dim=1)
            blocks[b.key] = v
        return blocks

    first, second = split(left), split(right)
    out = {}
    for p in plan.paths:
        copies = plan.block_by_key[p.key3].parity_copies
        a, b = first[p.key1][:, :copies], second[p.key2][:, :copies]
        comps = [None] * (1 if p.key3[0] == "scalar" else 2)
        for i, j, k, s in p.terms:
            term = (s * mags[p.cls]) * a[..., i] * b[..., j]
            comps[k] = term if comps[k] is None else comps[k] + term
        value = torch.stack(comps, -1) * weight[p.weight_start:p.weight_stop].view(
            1, copies, C, 1)
        out[p.key3] = value if p.key3 not in out else out[p.key3] + value
    pieces = []
    for b in plan.blocks:
        v = out.get(b.key)
        if v is None:
            v = left.new_zeros(n, b.parity_copies, C, b.irrep_dimension)
        if b.parity_copies == 2:
            v = torch.cat((v[:, :1], torch.stack((v[:, 1, :, 1], -v[:, 1, :, 0]), -1)[:, None]),
                          dim=1)
        pieces.append(v.reshape(n, -1))
    return torch.cat(pieces, dim=-1)


def _tp_backward_setup(ctx, inputs, output):
    left, right, weight, grad_output, channels, m_max, parity, normalization = inputs
    ctx.save_for_backward(left, right, weight, grad_output)
    ctx.config = (channels, m_max, parity, normalization)
    ctx.set_materialize_grads(False)


def _tp_double_backward(ctx, dd_left, dd_right, dd_weight):
    left, right, weight, grad_output = ctx.saved_tensors
    selected = [(i, c) for i, c in enumerate((dd_left, dd_right, dd_weight)) if c is not None]
    if not selected:
        return (None,) * 8
    plan = tp_plan(*ctx.config)
    with torch.enable_grad():
        operands = tuple(v.detach().requires_grad_(True)
                         for v in (left, right, weight, grad_output))
        value = torch_tp_flat(*operands[:3], plan)
        first = torch.autograd.grad(value, operands[:3], operands[3], create_graph=True)
        second = torch.autograd.grad(tuple(first[i] for i, _ in selected), operands,
                                     grad_outputs=tuple(c for _, c in selected),
                                     allow_unused=True)
    return (*second, None, None, None, None)


tp_backward.register_autograd(_tp_double_backward, setup_context=_tp_backward_setup)


# ---------------------------------------------------------------------- uvu ops


@torch.library.custom_op(f"{NAMESPACE}::uvu_forward", mutates_args=())
def uvu_forward(left: Tensor, right: Tensor, weight: Tensor, table: Tensor, config: list[int],
                shared: bool) -> Tensor:
    """out[N, width1] of UvuTensorProduct (reference uvu_triton.py:235-275)."""
    require_cuda_float32("UvuTensorProduct", left, right, weight)
    left, right, weight = left.contiguous(), right.contiguous(), weight.contiguous()
    out = torch.empty_like(left)
    with torch.cuda.device(left.device):
        fwd, _ = _lib.uvu_workspace(config, shared, left.shape[0], left.device)
        workspace = torch.empty(max(fwd, 16), dtype=torch.uint8, device=left.device)
        _lib.uvu_forward(left, right, weight, out, config, shared, table, workspace)
    return out


@uvu_forward.register_fake
def _uvu_forward_fake(left, right, weight, table, config, shared):
    return torch.empty_like(left)


@torch.library.custom_op(f"{NAMESPACE}::uvu_backward", mutates_args=())
def uvu_backward(left: Tensor, right: Tensor, weight: Tensor, grad_output: Tensor, table: Tensor,
                 config: list[int], shared: bool, needed: int
                 ) -> tuple[Tensor, Tensor, Tensor]:
    """(gx, gy, gw) for the roles in `needed` (1 = x, 2 = y, 4 = w); absent roles
    are empty (reference uvu_triton.py:287-404)."""
    require_cuda_float32("UvuTensorProduct backward", left, right, weight, grad_output)
    left, right = left.contiguous(), right.contiguous()
    weight, grad_output = weight.contiguous(), grad_output.contiguous()
    gx = torch.empty_like(left) if needed & 1 else left.new_empty(0)
    gy = torch.empty_like(right) if needed & 2 else right.new_empty(0)
    gw = torch.empty_like(weight) if needed & 4 else weight.new_empty(0)
    with torch.cuda.device(left.device):
        _, bwd = _lib.uvu_workspace(config, shared, left.shape[0], left.device)
        workspace = torch.empty(max(bwd, 16), dtype=torch.uint8, device=left.device)
        _lib.uvu_backward(left, right, weight, grad_output, gx if needed & 1 else None,
                          gy if needed & 2 else None, gw if needed & 4 else None, config, shared,
                          needed, table, workspace)
    return gx, gy, gw


@uvu_backward.register_fake
def _uvu_backward_fake(left, right, weight, grad_output, table, config, shared, needed):
    return (torch.empty_like(left) if needed & 1 else left.new_empty(0),
            torch.empty_like(right) if needed & 2 else right.new_empty(0),
            torch.empty_like(weight) if needed & 4 else weight.new_empty(0))


def _uvu_setup(ctx, inputs, output):
    left, right, weight, table, config, shared = inputs
    ctx.save_for_backward(left, right, weight, table)
    ctx.config, ctx.shared = config, shared


def _uvu_autograd(ctx, grad_output):
    left, right, weight, table = ctx.saved_tensors
    flags = ctx.needs_input_grad[:3]
    needed = sum(int(f) << i for i, f in enumerate(flags))
    if needed == 0:
        return None, None, None, None, None, None
    gx, gy, gw = uvu_backward(left, right, weight, grad_output.contiguous(), table, ctx.config,
                              ctx.shared, needed)
    return (gx if flags[0] else None, gy if flags[1] else None, gw if flags[2] else None,
            None, None, None)


uvu_forward.register_autograd(_uvu_autograd, setup_context=_uvu_setup)


def torch_uvu_flat(left: Tensor, right: Tensor, weight: Tensor, entries_in1, entries_in2,
                   paths, coefficients: Tensor, channels: int, channels_in2: int,
                   shared: bool) -> Tensor:
    """Differentiable PyTorch formula of the uvu map (the role of the reference's
    torch_uvu_forward, uvu_o2.py:50-73); used for second derivatives only."""
    rows = left.shape[0]
    values = [None] * len(entries_in1)
    for p, (i, j, k) in enumerate(paths):
        a, b, out = entries_in1[i], entries_in2[j], entries_in1[k]
        x = left[:, a.offset:a.offset + channels * a.dim].reshape(rows, channels, a.dim)
        y = right[:, b.offset:b.offset + channels_in2 * b.dim].reshape(rows, channels_in2, b.dim)
        start = p * channels * channels_in2
        w = weight[..., start:start + channels * channels_in2]
        if shared:
            projected = torch.einsum("uv,nvj->nuj", w.reshape(channels, channels_in2), y)
        else:
            projected = torch.einsum("nuv,nvj->nuj", w.reshape(rows, channels, channels_in2), y)
        cg = coefficients[p, :out.dim, :a.dim, :b.dim]
        contribution = torch.einsum("nui,nuj,kij->nuk", x, projected, cg)
        values[k] = contribution if values[k] is None else values[k] + contribution
    return torch.cat([value.reshape(rows, channels * entry.dim)
                      for entry, value in zip(entries_in1, values)], dim=-1)


# -------------------------------------------------------------------- radial ops


@torch.library.custom_op(f"{NAMESPACE}::radial_forward", mutates_args=())
def radial_forward(left: Tensor, angular: Tensor, hidden: Tensor, alpha: Tensor, bias: Tensor,
                   table: Tensor, rconfig: list[int], has_bias: bool) -> Tensor:
    """uvu(left, angular, hidden @ alpha^T + bias) with the edge weights regenerated
    on chip (reference radial_streamed.py:81-99)."""
    require_cuda_float32("RadialUvuTensorProduct", left, angular, hidden, alpha)
    left, angular = left.contiguous(), angular.contiguous()
    hidden, alpha = hidden.contiguous(), alpha.contiguous()
    bias = bias.contiguous() if has_bias else None
    out = torch.empty_like(left)
    with torch.cuda.device(left.device):
        fwd, _ = _lib.radial_workspace(rconfig, left.shape[0], left.device)
        workspace = torch.empty(max(fwd, 16), dtype=torch.uint8, device=left.device)
        _lib.radial_forward(left, angular, hidden, alpha, bias, out, rconfig, table, workspace)
    return out


@radial_forward.register_fake
def _radial_forward_fake(left, angular, hidden, alpha, bias, table, rconfig, has_bias):
    return torch.empty_like(left)


@torch.library.custom_op(f"{NAMESPACE}::radial_backward", mutates_args=())
def radial_backward(left: Tensor, angular: Tensor, hidden: Tensor, alpha: Tensor, bias: Tensor,
                    grad_output: Tensor, table: Tensor, rconfig: list[int], has_bias: bool,
                    needed: int) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """(g_left, g_angular, g_hidden, g_alpha, g_bias) for the role mask `needed`
    (1, 2, 4, 8, 16); absent roles are empty (reference radial_streamed.py:109-139)."""
    require_cuda_float32("RadialUvuTensorProduct backward", left, angular, hidden, alpha,
                         grad_output)
    left, angular = left.contiguous(), angular.contiguous()
    hidden, alpha, grad_output = hidden.contiguous(), alpha.contiguous(), grad_output.contiguous()
    if not has_bias:
        needed &= ~16
    bias_c = bias.contiguous() if has_bias else None
    # left and angular gradients come from one kernel; alpha's buffer is scratch for bias
    want_xy = bool(needed & 3)
    gx = torch.empty_like(left) if want_xy else left.new_empty(0)
    gy = torch.empty_like(angular) if want_xy else angular.new_empty(0)
    gh = torch.empty_like(hidden) if needed & 4 else hidden.new_empty(0)
    ga = torch.empty_like(alpha) if needed & 24 else alpha.new_empty(0)
    gb = torch.empty_like(bias) if needed & 16 else alpha.new_empty(0)
    kernel_mask = needed | (3 if want_xy else 0) | (8 if needed & 16 else 0)
    with torch.cuda.device(left.device):
        _, bwd = _lib.radial_workspace(rconfig, left.shape[0], left.device)
        workspace = torch.empty(max(bwd, 16), dtype=torch.uint8, device=left.device)
        _lib.radial_backward(left, angular, hidden, alpha, bias_c, grad_output,
                             gx if want_xy else None, gy if want_xy else None,
                             gh if needed & 4 else None, ga if needed & 24 else None,
                             gb if needed & 16 else None, rconfig, kernel_mask, table, workspace)
    return (gx if needed & 1 else left.new_empty(0), gy if needed & 2 else angular.new_empty(0),
            gh, ga if needed & 8 else alpha.new_empty(0), gb)


@radial_backward.register_fake
def _radial_backward_fake(left, angular, hidden, alpha, bias, grad_output, table, rconfig,
                          has_bias, needed):
    if not has_bias:
        needed &= ~16
    return (torch.empty_like(left) if needed & 1 else left.new_empty(0),
            torch.empty_like(angular) if needed & 2 else angular.new_empty(0),
            torch.empty_like(hidden) if needed & 4 else hidden.new_empty(0),
            torch.empty_like(alpha) if needed & 8 else alpha.new_empty(0),
            torch.empty_like(bias) if needed & 16 else alpha.new_empty(0))


def _radial_setup(ctx, inputs, output):
    left, angular, hidden, alpha, bias, table, rconfig, has_bias = inputs
    ctx.save_for_backward(left, angular, hidden, alpha, bias, table)
    ctx.rconfig, ctx.has_bias = rconfig, has_bias


def _radial_autograd(ctx, grad_output):
    left, angular, hidden, alpha, bias, table = ctx.saved_tensors
    flags = list(ctx.needs_input_grad[:5])
    if not ctx.has_bias:
        flags[4] = False
    needed = sum(int(f) << i for i, f in enumerate(flags))
    if needed == 0:
        return (None,) * 8
    grads = radial_backward(left, angular, hidden, alpha, bias, grad_output.contiguous(), table,
                            ctx.rconfig, ctx.has_bias, needed)
    return (*(g if f else None for g, f in zip(grads, flags)), None, None, None)


radial_forward.register_autograd(_radial_autograd, setup_context=_radial_setup)
