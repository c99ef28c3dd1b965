"""TensorProduct: the drop-in module over the fused sm_100a kernels.

Mirrors the reference's public class (src/ictc_o2_hp/api.py:18-29 over
triton_o2.py:1095-1201): constructor arguments, ``weight``,
``representation_dimension``, ``paths``, ``blocks``, ``keys``, ``parameter_count``,
``representation_spec()``, ``copy_weights_to_r5``/``load_weights_from_r5`` and the
state_dict keys (``weight``, ``cg_<p>``, ``odd_to_even``, ``even_to_odd``).
Weight initialisation consumes the global torch RNG exactly like the reference
(one ``torch.randn(out_mul) * 0.02`` per path, native_o2.py:110-117), so a seeded
construction yields identical weights.

Difference from the reference: non-CUDA or non-float32 operands raise instead of
falling back to PyTorch (no CPU path in this implementation).
"""

from __future__ import annotations

import torch

from . import ops
from ._algebra import RepresentationBlock, TpPlan, cg_tensor


def _validate(channels, m_max):
    """api.py:11-15."""
    if int(channels) != channels or channels < 1:
        raise ValueError("channels must be a positive integer")
    if int(m_max) != m_max or m_max < 0:
        raise ValueError("m_max must be a nonnegative integer")


class _TensorProductBase(torch.nn.Module):
    def __init__(self, channels, m_max, *, parity="full", normalization="component"):
        _validate(channels, m_max)
        super().__init__()
        if parity not in ("canonical", "full"):
            raise ValueError(parity)
        if normalization not in ("component", "norm"):
            raise ValueError(normalization)
        self.channels = int(channels)
        self.max_frequency = int(m_max)
        self.parity = parity
        self.normalization = normalization
        self._plan = TpPlan(self.channels, self.max_frequency, parity, normalization)
        self.blocks: tuple[RepresentationBlock, ...] = self._plan.blocks
        self.keys = self._plan.keys
        self.block_by_key = self._plan.block_by_key
        self.paths = tuple((p.key1, p.key2, p.key3) for p in self._plan.paths)
        self._weight_offsets = tuple((p.weight_start, p.weight_stop) for p in self._plan.paths)
        initial = []
        for p in self._plan.paths:
            initial.append(torch.randn(p.weight_stop - p.weight_start) * 0.02)
        for index, p in enumerate(self._plan.paths):
            cg = torch.from_numpy(cg_tensor(p.key1, p.key2, p.key3, normalization))
            self.register_buffer(f"cg_{index}", cg.contiguous(), persistent=True)
        j = torch.tensor([[0.0, -1.0], [1.0, 0.0]], dtype=torch.float64)
        self.register_buffer("odd_to_even", j.transpose(0, 1).contiguous(), persistent=True)
        self.register_buffer("even_to_odd", j.contiguous(), persistent=True)
        self.weight = torch.nn.Parameter(torch.cat(initial) if initial else torch.zeros(0))

    # --- reference attributes (native_o2.py:137-165, fast_o2.py:173-186)
    @property
    def representation_dimension(self) -> int:
        return self._plan.representation_dimension

    @property
    def parameter_count(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def representation_spec(self) -> list[dict]:
        rows = []
        for block in self.blocks:
            if block.frequency == 0:
                labels = block.token
            elif self.parity == "canonical":
                labels = str(block.frequency)
            else:
                labels = f"{block.frequency}e+{block.frequency}o"
            rows.append({"labels": labels, "frequency": block.frequency,
                         "irrep_dimension": block.irrep_dimension,
                         "multiplicity": block.multiplicity,
                         "parity_copies": block.parity_copies})
        return rows

    def copy_weights_to_r5(self, reference) -> None:
        """Copies the packed weight into a per-path reference operator."""
        if len(reference.weights) != len(self._weight_offsets):
            raise ValueError("r5 path count differs")
        with torch.no_grad():
            for parameter, (start, end) in zip(reference.weights, self._weight_offsets):
                parameter.copy_(self.weight[start:end])

    def load_weights_from_r5(self, reference) -> None:
        """Copies a per-path reference operator's weights into the packed layout."""
        if len(reference.weights) != len(self._weight_offsets):
            raise ValueError("r5 path count differs")
        with torch.no_grad():
            for parameter, (start, end) in zip(reference.weights, self._weight_offsets):
                self.weight[start:end].copy_(parameter)

    def _flat(self, left: torch.Tensor, right: torch.Tensor, layout: int = 0) -> torch.Tensor:
        width = self.representation_dimension
        out = ops.tp_forward(left.reshape(-1, width), right.reshape(-1, width), self.weight,
                             self.channels, self.max_frequency, self.parity, self.normalization,
                             layout)
        return out


class TensorProduct(_TensorProductBase):
    """Flat channel-major O(2) product with all path weights trainable.

    Inputs/outputs: ``(*batch, representation_dimension)``; positive-frequency
    blocks use ``[copy, channel, component]`` (full) or ``[channel, component]``
    (canonical); the full second copy keeps its reflection-twisted basis.
    """

    def forward(self, left: torch.Tensor, right: torch.Tensor) -> torch.Tensor:
        if (left.ndim < 1 or left.shape[-1] != self.representation_dimension
                or right.shape != left.shape):
            raise ValueError("flat O(2) inputs must have the configured width")
        return self._flat(left, right).reshape(left.shape)


class TupleTensorProduct(_TensorProductBase):
    """One ``(*batch, multiplicity, irrep_dimension)`` tensor per block in and out
    (reference: api.py:32-37, triton_o2.py:1134-1166)."""

    def forward(self, left, right):
        if len(left) != len(self.keys) or len(right) != len(self.keys):
            raise ValueError("one tensor per representation block is required")
        batch = left[0].shape[:-2]
        flat_l = torch.cat([v.reshape(*batch, -1) for v in left], dim=-1)
        flat_r = torch.cat([v.reshape(*batch, -1) for v in right], dim=-1)
        out = self._flat(flat_l, flat_r).reshape(*batch, -1)
        pieces, cursor = [], 0
        for block in self.blocks:
            width = block.multiplicity * block.irrep_dimension
            pieces.append(out[..., cursor:cursor + width].reshape(
                *batch, block.multiplicity, block.irrep_dimension))
            cursor += width
        return tuple(pieces)


class ComponentMajorTensorProduct(_TensorProductBase):
    """Flat product with ``[copy, component, channel]`` frequency blocks (reference:
    api.py:40-49, triton_o2.py:1204-1278).  Storage order only: the full-parity
    second copy keeps the reflection-twisted basis."""

    def _to_channel_major(self, value):
        batch = value.shape[:-1]
        pieces, cursor = [], 0
        for block in self.blocks:
            width = block.multiplicity * block.irrep_dimension
            part = value[..., cursor:cursor + width]
            if block.irrep_dimension == 2:
                part = part.reshape(*batch, block.parity_copies, 2, self.channels)
                part = part.transpose(-1, -2).reshape(*batch, width)
            pieces.append(part)
            cursor += width
        return torch.cat(pieces, dim=-1)

    def _to_component_major(self, value):
        batch = value.shape[:-1]
        pieces, cursor = [], 0
        for block in self.blocks:
            width = block.multiplicity * block.irrep_dimension
            part = value[..., cursor:cursor + width]
            if block.irrep_dimension == 2:
                part = part.reshape(*batch, block.parity_copies, self.channels, 2)
                part = part.transpose(-1, -2).reshape(*batch, width)
            pieces.append(part)
            cursor += width
        return torch.cat(pieces, dim=-1)

    def forward(self, left, right):
        if (left.ndim < 1 or left.shape[-1] != self.representation_dimension
                or right.shape != left.shape):
            raise ValueError("flat O(2) inputs must have the configured width")
        # the kernels address component-major frequency blocks in place (the
        # reference's layout-1/2 metadata, triton_o2.py:114-118)
        return self._flat(left, right, layout=1).reshape(left.shape)
