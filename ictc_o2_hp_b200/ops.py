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
               parity: str, normalization: str, layout: int = 0) -> Tensor:
    """out[N, W] of TensorProduct on flat rows (triton_o2.py:786-875); layout 1 reads
    and writes component-major frequency blocks in place."""
    require_cuda_float32("TensorProduct", left, right, weight)
    left, right, weight = left.contiguous(), right.contiguous(), weight.contiguous()
    out = torch.empty_like(left)
    with torch.cuda.device(left.device):
        _lib.tp_forward(left, right, weight, out, channels, m_max, parity, normalization, layout)
    return out


@tp_forward.register_fake
def _tp_forward_fake(left, right, weight, channels, m_max, parity, normalization, layout=0):
    return torch.empty_like(left)


@torch.library.custom_op(f"{NAMESPACE}::tp_backward", mutates_args=())
def tp_backward(left: Tensor, right: Tensor, weight: Tensor, grad_output: Tensor, channels: int,
                m_max: int, parity: str, normalization: str, layout: int = 0
                ) -> tuple[Tensor, Tensor, Tensor]:
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
                         workspace, channels, m_max, parity, normalization, layout)
    return grad_left, grad_right, grad_weight


@tp_backward.register_fake
def _tp_backward_fake(left, right, weight, grad_output, channels, m_max, parity, normalization,
                      layout=0):
    return torch.empty_like(left), torch.empty_like(right), torch.empty_like(weight)


def _tp_setup(ctx, inputs, output):
    left, right, weight, channels, m_max, parity, normalization, layout = inputs
    ctx.save_for_backward(left, right, weight)
    ctx.config = (channels, m_max, parity, normalization, layout)


def _tp_autograd(ctx, grad_output):
    left, right, weight = ctx.saved_tensors
    gx, gy, gw = tp_backward(left, right, weight, grad_output.contiguous(), *ctx.config)
    return gx, gy, gw, None, None, None, None, None


tp_forward.register_autograd(_tp_autograd, setup_context=_tp_setup)


def torch_tp_flat(left: Tensor, right: Tensor, weight: Tensor, plan: TpPlan) -> Tensor:
    """Differentiable PyTorch formula of the same map (the role of
    triton_o2.py:969-1032); run in float64 on the CPU it is the reference the
    second-derivative tests check the kernels against."""
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
    left, right, weight, grad_output, channels, m_max, parity, normalization, layout = inputs
    ctx.save_for_backward(left, right, weight, grad_output)
    ctx.config = (channels, m_max, parity, normalization, layout)
    ctx.set_materialize_grads(False)


def _accumulate(total, term):
    return term if total is None else total + term


def _tp_double_backward(ctx, dd_left, dd_right, dd_weight):
    """Second derivatives through the same kernels (the reference recomputes them in
    PyTorch, triton_o2.py:1041-1069).  With B(x, y; w) the trilinear map and
    dx = B_x^T(g; y, w), dy = B_y^T(g; x, w), dw = B_w^T(g; x, y), the cotangents
    (ddx, ddy, ddw) contract to <B(ddx, y; w) + B(x, ddy; w) + B(x, y; ddw), g>, so
      d left   = B_x^T(g; ddy, w) + B_x^T(g; y, ddw)
      d right  = B_y^T(g; ddx, w) + B_y^T(g; x, ddw)
      d weight = B_w^T(g; ddx, y) + B_w^T(g; x, ddy)
      d g      = B(ddx, y; w) + B(x, ddy; w) + B(x, y; ddw):
    three backward calls (operands swapped in) and up to three forward calls."""
    left, right, weight, grad_output = ctx.saved_tensors
    cfg = ctx.config
    need_x, need_y, need_w, need_g = ctx.needs_input_grad[:4]
    d_left = d_right = d_weight = d_g = None
    if dd_left is not None and (need_y or need_w):
        _, gy, gw = tp_backward(dd_left, right, weight, grad_output, *cfg)
        d_right = gy if need_y else None
        d_weight = gw if need_w else None
    if dd_right is not None and (need_x or need_w):
        gx, _, gw = tp_backward(left, dd_right, weight, grad_output, *cfg)
        if need_x:
            d_left = _accumulate(d_left, gx)
        if need_w:
            d_weight = _accumulate(d_weight, gw)
    if dd_weight is not None and (need_x or need_y):
        gx, gy, _ = tp_backward(left, right, dd_weight, grad_output, *cfg)
        if need_x:
            d_left = _accumulate(d_left, gx)
        if need_y:
            d_right = _accumulate(d_right, gy)
    if need_g:
        if dd_left is not None:
            d_g = _accumulate(d_g, tp_forward(dd_left, right, weight, *cfg))
        if dd_right is not None:
            d_g = _accumulate(d_g, tp_forward(left, dd_right, weight, *cfg))
        if dd_weight is not None:
            d_g = _accumulate(d_g, tp_forward(left, right, dd_weight, *cfg))
    return d_left, d_right, d_weight, d_g, None, None, None, None, None


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
    torch_uvu_forward, uvu_o2.py:50-73); run in float64 on the CPU it is the
    reference the second-derivative tests check the kernels against."""
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


def _radial_backward_setup(ctx, inputs, output):
    left, angular, hidden, alpha, bias, grad_output, table, rconfig, has_bias, needed = inputs
    ctx.save_for_backward(left, angular, hidden, alpha, bias, grad_output, table)
    ctx.rconfig, ctx.has_bias = rconfig, has_bias
    ctx.set_materialize_grads(False)


def _radial_double_backward(ctx, d_left, d_angular, d_hidden, d_alpha, d_bias):
    """Second derivatives through the same kernels (reference
    radial_streamed.py:173-207).  With out = F(x, y, r, a) + G(x, y, b) (F the
    product with the regenerated weights r a^T, G the one with the bias), each
    cotangent contracts with its gradient to <product with that operand swapped in,
    g>: <dx, gx> = <out(dx, y, r, a, b), g>, <dr, gr> = <F(x, y, dr, a), g>,
    <da, ga> + <db, gb> = <out(x, y, r, da, db), g>.  Each term is one role-masked
    backward call for the other operands and one forward call for g."""
    left, angular, hidden, alpha, bias, grad_output, table = ctx.saved_tensors
    need = list(ctx.needs_input_grad[:6])
    if not ctx.has_bias:
        need[4] = False
    acc = [None] * 6
    empty = alpha.new_empty(0)

    def add(operands, roles, has_bias):
        selected = [r for r in roles if need[r] and (r != 4 or has_bias)]
        if selected:
            mask = sum(1 << r for r in selected)
            grads = radial_backward(*operands, grad_output, table, ctx.rconfig, has_bias, mask)
            for r in selected:
                acc[r] = grads[r] if acc[r] is None else acc[r] + grads[r]
        if need[5]:
            value = radial_forward(*operands, table, ctx.rconfig, has_bias)
            acc[5] = value if acc[5] is None else acc[5] + value

    bias_operand = bias if ctx.has_bias else empty
    if d_left is not None and d_left.numel():
        add((d_left, angular, hidden, alpha, bias_operand), (1, 2, 3, 4), ctx.has_bias)
    if d_angular is not None and d_angular.numel():
        add((left, d_angular, hidden, alpha, bias_operand), (0, 2, 3, 4), ctx.has_bias)
    if d_hidden is not None and d_hidden.numel():
        add((left, angular, d_hidden, alpha, empty), (0, 1, 3), False)
    has_da = d_alpha is not None and d_alpha.numel() > 0
    has_db = ctx.has_bias and d_bias is not None and d_bias.numel() > 0
    if has_da or has_db:
        add((left, angular, hidden, d_alpha if has_da else torch.zeros_like(alpha),
             d_bias if has_db else empty), (0, 1, 2), has_db)
    return (*acc, None, None, None, None)


radial_backward.register_autograd(_radial_double_backward, setup_context=_radial_backward_setup)
