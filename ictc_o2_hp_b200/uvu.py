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

from functools import lru_cache

import numpy as np
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


@lru_cache(maxsize=None)
def uvu_plan(channels, channels_in2, m_max, parity, m_max_in2, parity_in2, normalization,
             path_normalization):
    """(entries_in1, entries_in2, paths, coefficients) of a configuration."""
    _, e1, _ = uvu_representation(channels, m_max, parity)
    _, e2, _ = uvu_representation(channels_in2, m_max_in2, parity_in2)
    paths, coef = uvu_paths(e1, e2, normalization, path_normalization, channels_in2)
    return e1, e2, paths, coef


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
    ctx.save_for_backward(left, right, weight, grad_output)
    ctx.config, ctx.shared = config, shared
    ctx.set_materialize_grads(False)


def _uvu_double_backward(ctx, dd_left, dd_right, dd_weight):
    """Second derivatives through the differentiable PyTorch formula (the role of
    uvu_triton.py:442-457)."""
    left, right, weight, grad_output = ctx.saved_tensors
    selected = [(i, c) for i, c in enumerate((dd_left, dd_right, dd_weight))
                if c is not None and c.numel()]
    if not selected:
        return (None,) * 8
    inv_parity = {v: k for k, v in PARITY_CODE.items()}
    inv_norm = {v: k for k, v in NORM_CODE.items()}
    c = ctx.config
    e1, e2, paths, coef = uvu_plan(c[0], c[1], c[2], inv_parity[c[3]], c[4], inv_parity[c[5]],
                                   inv_norm[c[6]], "path" if c[7] else "none")
    coefficients = torch.from_numpy(np.asarray(coef)).to(left)
    with torch.enable_grad():
        operands = tuple(v.detach().requires_grad_(True)
                         for v in (left, right, weight, grad_output))
        value = ops.torch_uvu_flat(operands[0], operands[1], operands[2], e1, e2, paths,
                                   coefficients, c[0], c[1], ctx.shared)
        first = torch.autograd.grad(value, operands[:3], operands[3], create_graph=True)
        second = torch.autograd.grad(tuple(first[i] for i, _ in selected), operands,
                                     grad_outputs=tuple(cot for _, cot in selected),
                                     allow_unused=True)
    return (*second, None, None, None, None)


ops.uvu_backward.register_autograd(_uvu_double_backward, setup_context=_uvu_backward_setup)
