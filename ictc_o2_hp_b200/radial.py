"""RadialUvuTensorProduct: a radial network's final affine layer fused with a V=1
per-edge uvu product over the sm_100a kernels.

Mirrors the reference class (src/ictc_o2_hp/radial_uvu.py:21-66): equivalent to
``tp(left, angular, radial_out(radial_hidden))`` with the constructor checks of the
reference; the supplied ``torch.nn.Linear`` is reused unchanged (state_dict keys
``tp.weight``, ``radial_out.weight``, ``radial_out.bias``).  The edge weights are
regenerated on chip instead of being materialised.  Non-CUDA or non-float32
operands raise instead of falling back.
"""

from __future__ import annotations

import torch

from . import ops
from .uvu import UvuTensorProduct


class RadialUvuTensorProduct(torch.nn.Module):
    """Equivalent to ``tp(left, angular, radial_out(radial_hidden))``."""

    def __init__(self, tp: UvuTensorProduct, radial_out: torch.nn.Linear):
        super().__init__()
        if not isinstance(tp, UvuTensorProduct):
            raise TypeError("tp must be an O(2) uvu tensor product")
        if tp.channels_in2 != 1 or tp.shared_weights or tp.internal_weights:
            raise ValueError("radial fusion requires V=1 and external per-edge TP weights")
        if not isinstance(radial_out, torch.nn.Linear):
            raise TypeError("radial_out must be the final torch.nn.Linear of the radial network")
        if radial_out.out_features != tp.weight_numel:
            raise ValueError("radial_out.out_features must equal tp.weight_numel")
        if radial_out.in_features < 1:
            raise ValueError("radial_out must have at least one input feature")
        self.tp = tp
        self.radial_out = radial_out

    def _rconfig(self):
        c = self.tp._config
        return [c[0], c[2], c[3], c[4], c[5], c[6], c[7], self.radial_out.in_features]

    def forward(self, left, angular, radial_hidden):
        tp = self.tp
        if left.ndim < 1 or left.shape[-1] != tp.input1_dimension:
            raise ValueError("left has the wrong final dimension")
        if angular.shape != (*left.shape[:-1], tp.input2_dimension):
            raise ValueError("angular must have the same batch shape and configured dimension")
        if radial_hidden.shape != (*left.shape[:-1], self.radial_out.in_features):
            raise ValueError(
                "radial_hidden must have the same batch shape and affine input dimension")
        if not left.is_floating_point():
            raise TypeError("radial uvu operands must be real floating-point tensors")
        operands = [angular, radial_hidden, self.radial_out.weight, tp._coefficients]
        if self.radial_out.bias is not None:
            operands.append(self.radial_out.bias)
        if any(v.device != left.device or v.dtype != left.dtype for v in operands):
            raise ValueError("all operands and modules must have the same device and dtype")
        bias = self.radial_out.bias
        has_bias = bias is not None
        out = ops.radial_forward(
            left.reshape(-1, tp.input1_dimension), angular.reshape(-1, tp.input2_dimension),
            radial_hidden.reshape(-1, self.radial_out.in_features), self.radial_out.weight,
            bias if has_bias else self.radial_out.weight.new_empty(0), tp._table,
            self._rconfig(), has_bias)
        return out.reshape(*left.shape[:-1], tp.representation_dimension)
