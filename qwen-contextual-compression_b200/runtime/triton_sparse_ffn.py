"""Drop-in for reference runtime/triton_sparse_ffn.py: ``triton_indexed_ffn``.

The reference's batch-1 backend reads the selected weights indirectly with
two Triton kernels (runtime/triton_sparse_ffn.py:13-25) and checks its
arguments first (:28-35).  This module keeps the name, signature, checks and
error messages, and runs the same fused sm_100a kernel as ``cuda_indexed_ffn``
over the layer's packed records (built on first use and cached per weight
tensors).  No Triton is used: ``TRITON_AVAILABLE`` is False and the entry
point does not depend on it.
"""
from __future__ import annotations

from .cuda_indexed import _engine_for, validate_selected_ids

TRITON_AVAILABLE = False  # the fused CUDA kernel serves this entry point


def triton_indexed_ffn(x, selected_ids, gate_weight, up_weight, down_weight, transposed_down=False):
    """y [1, hidden] in x's dtype; never materialises K x H gathered matrices."""
    if not x.is_cuda:
        raise ValueError("triton_indexed requires CUDA tensors")
    if x.ndim != 2 or x.shape[0] != 1 or selected_ids.ndim != 1:
        raise ValueError("triton_indexed currently targets batch=1")
    hidden = x.shape[-1]
    intermediate = gate_weight.shape[0]
    expected = (intermediate, hidden) if transposed_down else (hidden, intermediate)
    if tuple(down_weight.shape) != expected:
        raise ValueError(f"down weight shape must be {expected} for transposed_down={transposed_down}")
    validate_selected_ids(selected_ids, intermediate)
    if x.dtype != gate_weight.dtype:
        raise RuntimeError(f"x dtype {x.dtype} must match the weight dtype {gate_weight.dtype}")
    engine = _engine_for(gate_weight, up_weight, down_weight, transposed_down)
    return engine(x, selected_ids)


__all__ = ["TRITON_AVAILABLE", "triton_indexed_ffn"]
