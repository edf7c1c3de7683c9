"""Module-style drop-in for reference runtime/ffn.py's dynamic sparse FFN.

``TorchDynamicSparseFFN(gate, up, down)(x, selected_ids)`` keeps the
reference constructor and call (runtime/ffn.py:34-39): weights gate/up [N,H]
and down [H,N], a 1-D id list shared by every row of x.  Instead of three
``index_select`` gathers and three GEMVs it packs the layer once into
neuron-major records and runs the fused kernel.  CUDA tensors only.
"""
from __future__ import annotations

import torch
from torch import nn

from .engine import IndexedSparseFFN
from .packing import pack_neuron_major, validate_weight_shapes


class TorchDynamicSparseFFN(nn.Module):
    """Selected-before-gate sparse FFN; same arguments as runtime/ffn.py:34-39."""

    def __init__(self, gate_weight: torch.Tensor, up_weight: torch.Tensor, down_weight: torch.Tensor,
                 transposed_down: bool = False, check_bounds: bool = False):
        super().__init__()
        validate_weight_shapes(gate_weight, up_weight, down_weight, transposed_down)
        self.engine = IndexedSparseFFN(pack_neuron_major(gate_weight, up_weight, down_weight, transposed_down),
                                       check_bounds=check_bounds)

    @property
    def hidden(self) -> int:
        return self.engine.hidden

    @property
    def intermediate(self) -> int:
        return self.engine.intermediate

    def activations(self, x: torch.Tensor, selected_ids: torch.Tensor) -> torch.Tensor:
        """a = silu(x G_sel^T) * (x U_sel^T), [B, K] in x dtype (the third item of the
        reference's ``components``)."""
        x2 = x if x.ndim == 2 else x.unsqueeze(0)
        activation = torch.empty((x2.shape[0], selected_ids.numel()), dtype=x.dtype, device=x.device)
        self.engine(x2, selected_ids, activation=activation)
        return activation

    def forward(self, x: torch.Tensor, selected_ids: torch.Tensor) -> torch.Tensor:
        if selected_ids.ndim != 1:
            raise ValueError("batch-1 sparse runtime requires one-dimensional selected_ids")
        return self.engine(x, selected_ids)
