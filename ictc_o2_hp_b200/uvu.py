"""UvuTensorProduct: O(2) products preserving the first input channel and summing the
second, over the sm_100a uvu kernels.

Mirrors the reference's public class (src/ictc_o2_hp/uvu_o2.py:76-240): constructor
arguments and validation, ``entries_in1/in2/out``, ``paths``, ``weight_numel``,
``weight_shape``, ``input1_dimension``, ``input2_dimension``,
``representation_dimension``, ``parameter_count``, ``weight_view_for_path`` and the
``weight`` parameter (``torch.randn(weight_numel) * 0.02`` for internal weights,
uvu_o2.py:153-156).  Non-CUDA or non-float32 operands raise instead of falling back.
"""

from __future__ import annotations

import torch

from . import _lib, ops
from ._algebra import uvu_paths, uvu_representation

PARITY_CODE = {"canonical": 0, "full": 1}
NORM_CODE = {"component": 0, "norm": 1}


def _integer(value, name, minimum):
    """uvu_o2.py:21-24."""
    if isinstance(value, bool) or int(value) != value or value < minimum:
        raise ValueError(f"{name} must be an integer >= {minimum}")
    return int(value)


class UvuTensorProduct(torch.nn.Module):
    """Flat Cartesian O(2) uvu product on CUDA FP32.

    ``output[k, u] += sum_v weight[p, u, v] * CG(input1[i, u], input2[j, v])`` for every
    legal entry path p = (i, j, k); first input and output have ``channels`` per copy,
    the second input ``channels_in2``.  ``shared_weights=False`` takes a per-row
    ``(*batch, weight_numel)`` weight on each call.
    """

    connection_mode = "uvu"

    def __init__(self, channels, channels_in2, m_max, *, parity="full", parity_in2=None,
                 m_max_in2=None, normalization="component", path_normalization="none",
                 internal_weights=None, shared_weights=True):
        super().__init__()
        self.channels = _integer(channels, "channels", 1)
        self.channels_in2 = _integer(channels_in2, "channels_in2", 1)
        self.m_max = _integer(m_max, "m_max", 0)
        self.m_max_in2 = _integer(m_max if m_max_in2 is None else m_max_in2, "m_max_in2", 0)
        self.parity = parity
        self.parity_in2 = parity if parity_in2 is None else parity_in2
        if normalization not in ("component", "norm"):
            raise ValueError("normalization must be component or norm")
        if path_normalization not in ("none", "element", "path"):
            raise ValueError("path_normalization must be none, element or path")
        self.normalization, self.path_normalization = normalization, path_normalization
        self.shared_weights = bool(shared_weights)
        self.internal_weights = (self.shared_weights if internal_weights is None
                                 else bool(internal_weights))
        if self.internal_weights and not self.shared_weights:
            raise ValueError("internal_weights requires shared_weights=True")
        self.blocks, self.entries_in1, self.input1_dimension = uvu_representation(
            self.channels, self.m_max, self.parity)
        self.blocks_in2, self.entries_in2, self.input2_dimension = uvu_representation(
            self.channels_in2, self.m_max_in2, self.parity_in2)
        self.entries_out = self.entries_in1
        self.representation_dimension = self.input1_dimension
        self.keys = tuple(block.key for block in self.blocks)
        paths, coef = uvu_paths(self.entries_in1, self.entries_in2, normalization,
                                path_normalization, self.channels_in2)
        self.paths = paths
        self.weight_numel = len(paths) * self.channels * self.channels_in2
        self.weight_shape = (self.weight_numel,)
        self._coefficient_values = coef
        self.register_buffer("_coefficients", torch.from_numpy(coef).to(torch.get_default_dtype()),
                             persistent=False)
        self._config = [self.channels, self.channels_in2, self.m_max,
                        PARITY_CODE[self.parity], self.m_max_in2, PARITY_CODE[self.parity_in2],
                        NORM_CODE[normalization], int(path_normalization != "none")]
        table = _lib.uvu_table(self._config)
        self.register_buffer("_table", torch.from_numpy(table), persistent=False)
        if self.internal_weights:
            self.weight = torch.nn.Parameter(torch.randn(self.weight_numel) * 0.02)
        else:
            self.register_buffer("weight", torch.empty(0))

    @property
    def parameter_count(self):
        return self.weight.numel() if self.internal_weights else 0

    def _apply(self, fn, recurse=True):
        super()._apply(fn, recurse)
        # keep the exact coefficients when converting dtypes (uvu_o2.py:162-170)
        self._coefficients.copy_(torch.from_numpy(self._coefficient_values).to(
            dtype=self._coefficients.dtype, device=self._coefficients.device))
        return self

    def _prepare(self, left, right, weight):
        """uvu_o2.py:172-190."""
        if left.ndim < 1 or left.shape[-1] != self.input1_dimension:
            raise ValueError(f"left must end in input1_dimension={self.input1_dimension}")
        if (right.ndim < 1 or right.shape[-1] != self.input2_dimension
                or right.shape[:-1] != left.shape[:-1]):
            raise ValueError(
                "right must have the same batch shape and configured input2_dimension")
        if weight is None:
            if not self.internal_weights:
                raise ValueError("external weights are required")
            weight = self.weight
        expected = ((self.weight_numel,) if self.shared_weights
                    else (*left.shape[:-1], self.weight_numel))
        if weight.shape != expected:
            raise ValueError(f"weight shape must be {expected}")
        if not left.is_floating_point():
            raise TypeError("uvu inputs and weights must be real floating-point tensors")
        if any(value.device != left.device or value.dtype != left.dtype
               for value in (right, weight, self._coefficients)):
            raise ValueError("both inputs, weights and module must have the same device and dtype")
        return weight

    def weight_view_for_path(self, path, weight=None):
        """uvu_o2.py:192-202."""
        if not 0 <= path < len(self.paths):
            raise IndexError("invalid uvu path index")
        if weight is None:
            if not self.internal_weights:
                raise ValueError("external weights are required")
            weight = self.weight
        start = path * self.channels * self.channels_in2
        return weight[..., start:start + self.channels * self.channels_in2].reshape(
            *weight.shape[:-1], self.channels, self.channels_in2)

    def forward(self, left, right, weight=None):
        weight = self._prepare(left, right, weight)
        ops.require_cuda_float32("UvuTensorProduct", left, right, weight)
        flat_weight = weight if self.shared_weights else weight.reshape(-1, self.weight_numel)
        result = ops.uvu_forward(left.reshape(-1, self.input1_dimension),
                                 right.reshape(-1, self.input2_dimension), flat_weight,
                                 self._table, self._config, self.shared_weights)
        return result.reshape(*left.shape[:-1], self.representation_dimension)


def _uvu_backward_setup(ctx, inputs, output):
    left, right, weight, grad_output, table, config, shared, needed = inputs
    ctx.save_for_backward(left, right, weight, grad_output, table)
    ctx.config, ctx.shared = config, shared
    ctx.set_materialize_grads(False)


def _uvu_double_backward(ctx, dd_left, dd_right, dd_weight):
    """Second derivatives through the same kernels, with role-pruned backward calls
    (the reference recomputes them in PyTorch, uvu_triton.py:442-457).  The map is
    trilinear in (x, y, w); the cotangents (ddx, ddy, ddw) contract to
    <B(ddx, y; w) + B(x, ddy; w) + B(x, y; ddw), g>, so
      d left   = B_x^T(g; ddy, w) + B_x^T(g; y, ddw)
      d right  = B_y^T(g; ddx, w) + B_y^T(g; x, ddw)
      d weight = B_w^T(g; ddx, y) + B_w^T(g; x, ddy)
      d g      = B(ddx, y; w) + B(x, ddy; w) + B(x, y; ddw)."""
    left, right, weight, grad_output, table = ctx.saved_tensors
    cfg, shared = ctx.config, ctx.shared
    ddx, ddy, ddw = (c if c is not None and c.numel() else None
                     for c in (dd_left, dd_right, dd_weight))
    need_x, need_y, need_w, need_g = ctx.needs_input_grad[:4]
    terms = {0: [], 1: [], 2: []}

    def backward(x, y, w, roles):
        mask = sum(1 << r for r in roles)
        if mask:
            outs = ops.uvu_backward(x, y, w, grad_output, table, cfg, shared, mask)
            for r in roles:
                terms[r].append(outs[r])

    if ddx is not None:
        backward(ddx, right, weight, [r for r, n in ((1, need_y), (2, need_w)) if n])
    if ddy is not None:
        backward(left, ddy, weight, [r for r, n in ((0, need_x), (2, need_w)) if n])
    if ddw is not None:
        backward(left, right, ddw, [r for r, n in ((0, need_x), (1, need_y)) if n])
    d_g = None
    if need_g:
        for x, y, w in ((ddx, right, weight), (left, ddy, weight), (left, right, ddw)):
            if x is not None and y is not None and w is not None:
                value = ops.uvu_forward(x, y, w, table, cfg, shared)
                d_g = value if d_g is None else d_g + value
    grads = [None if not terms[r] else sum(terms[r][1:], terms[r][0]) for r in range(3)]
    return (*grads, d_g, None, None, None, None)


ops.uvu_backward.register_autograd(_uvu_double_backward, setup_context=_uvu_backward_setup)
