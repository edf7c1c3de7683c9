"""x-only oracle sparse MLP wrapper with the GPU selector on the hot path.

Same interface as reference end_to_end/oracle_sparse_mlp.py:35-98:
``OracleSparseMLP(original, layer_idx, retention=1.0, telemetry=None,
norm_chunk_columns=256)`` with ``forward(x)`` only, ``set_mode``,
``last_selected_indices``, ``down_column_norms``, ``norm_computation_count``
and ``close``.  A down_proj pre-hook scores the live activation as
|a| * ||D[:, j]||_2 (fp32), keeps the K = ceil(retention * N) best neurons
per row and zeroes the rest before the original dense down projection.

The selection runs on the qcc_b200 top-K kernel, which fixes the tie order
the reference leaves to torch.topk (ties go to the lower index); the
selected set equals the reference's whenever the K-th and (K+1)-th scores
differ.  ``last_selected_indices`` is int64 [rows, K], ascending.
"""
from __future__ import annotations

import math
from typing import Callable

import torch
from torch import Tensor, nn

from ..runtime.selector import select_topk


@torch.no_grad()
def compute_down_column_norms_chunked(weight: Tensor, chunk_columns: int = 256) -> Tensor:
    """fp32 L2 norms of the columns of down [H, N], converting at most chunk_columns at a time
    (reference end_to_end/oracle_sparse_mlp.py:10-32).  Returned on the weight's device."""
    if weight.ndim != 2:
        raise ValueError("down projection weight must be a matrix")
    if chunk_columns <= 0:
        raise ValueError("chunk_columns must be positive")
    if weight.device.type == "meta":
        raise RuntimeError("down projection is still meta; Accelerate did not materialize it before the pre-hook")
    width = weight.shape[1]
    norms = torch.empty(width, dtype=torch.float32, device=weight.device)
    for start in range(0, width, chunk_columns):
        end = min(start + chunk_columns, width)
        norms[start:end] = torch.linalg.vector_norm(weight.detach()[:, start:end].float(), ord=2, dim=0)
    return norms


def output_metrics(dense: Tensor, sparse: Tensor, eps: float = 1e-12) -> dict[str, Tensor]:
    """Cosine / relative L2 / MSE / max-abs per row (reference evaluation/metrics.py:18-23)."""
    dense, sparse = dense.float(), sparse.float()
    delta = dense - sparse
    denom = (torch.linalg.vector_norm(dense, dim=-1) * torch.linalg.vector_norm(sparse, dim=-1)).clamp_min(eps)
    cosine = ((dense * sparse).sum(-1) / denom).clamp(-1.0, 1.0)
    cosine = torch.where((dense == sparse).all(-1), torch.ones_like(cosine), cosine)
    return {"cosine_similarity": cosine,
            "relative_l2": torch.linalg.vector_norm(delta, dim=-1) / (torch.linalg.vector_norm(dense, dim=-1) + eps),
            "mse": delta.square().mean(-1), "max_absolute_error": delta.abs().amax(-1)}


class OracleSparseMLP(nn.Module):
    """Select neurons from the live activation of ``forward(x)`` only (no dense reference input)."""

    actual_oracle_executes_dense_gate_up = True
    runtime_speedup_claimed = False

    def __init__(self, original: nn.Module, layer_idx: int, retention: float = 1.0,
                 telemetry: Callable[[int, dict[str, Tensor]], None] | None = None,
                 norm_chunk_columns: int = 256):
        super().__init__()
        if norm_chunk_columns <= 0:
            raise ValueError("norm_chunk_columns must be positive")
        self.original = original
        self.layer_idx = layer_idx
        self.retention = float(retention)
        self.enabled = False
        self.telemetry = telemetry
        self.norm_chunk_columns = norm_chunk_columns
        self.norm_computation_count = 0
        self.norm_preparation_log = None
        self.last_selected_indices = None
        self._current_input = None
        self.register_buffer("down_column_norms", None, persistent=False)
        down = original.down_proj
        self._accelerate_old_forward = None
        self._norm_hook = None
        if hasattr(down, "_hf_hook") and hasattr(down, "_old_forward"):
            # Accelerate materialises offloaded weights inside its rewritten forward,
            # after ordinary pre-hooks: intercept the inner forward instead.
            self._accelerate_old_forward = down._old_forward

            def intercepted(*args, **kwargs):
                replacement = self._prepare_down(down, args)
                return self._accelerate_old_forward(*(replacement or args), **kwargs)

            self._accelerate_interceptor = intercepted
            down._old_forward = intercepted
        else:
            self._norm_hook = down.register_forward_pre_hook(self._prepare_down)

    @property
    def intermediate_size(self) -> int:
        return int(self.original.down_proj.weight.shape[1])

    def _prepare_down(self, module, args):
        if not self.enabled or self.retention >= 1.0:
            return None
        weight = module.weight
        if self.down_column_norms is None:
            self.down_column_norms = compute_down_column_norms_chunked(weight, self.norm_chunk_columns)
            self.norm_computation_count += 1
            self.norm_preparation_log = {
                "layer": self.layer_idx, "down_shape": list(weight.shape), "weight_dtype": str(weight.dtype),
                "weight_device": str(weight.device), "norm_chunk_columns": self.norm_chunk_columns,
                "estimated_fp32_temp_mib": weight.shape[0] * min(weight.shape[1], self.norm_chunk_columns) * 4 / 2**20,
                "cached_norm_bytes": self.down_column_norms.numel() * 4}
        activation = args[0]
        n = self.intermediate_size
        k = max(1, min(n, math.ceil(self.retention * n)))
        norms = self.down_column_norms.to(device=activation.device, dtype=torch.float32)
        scores = (activation.detach().abs().float() * norms).reshape(-1, n)
        ids = select_topk(scores, k).long().reshape(*activation.shape[:-1], k)
        self.last_selected_indices = ids
        sparse_activation = torch.zeros_like(activation).scatter_(-1, ids, activation.gather(-1, ids))
        if self.telemetry is not None:
            dense_out = torch.nn.functional.linear(activation, weight, module.bias)
            sparse_out = torch.nn.functional.linear(sparse_activation, weight, module.bias)
            metrics = output_metrics(dense_out.flatten(0, -2), sparse_out.flatten(0, -2))
            incoming = torch.linalg.vector_norm(self._current_input.float(), dim=-1).flatten().clamp_min(1e-12)
            self.telemetry(self.layer_idx, {
                **metrics,
                "ffn_over_residual": torch.linalg.vector_norm(dense_out.float(), dim=-1).flatten() / incoming,
                "ffn_error_over_residual":
                    torch.linalg.vector_norm((dense_out - sparse_out).float(), dim=-1).flatten() / incoming})
        return (sparse_activation,)

    def set_mode(self, enabled: bool, retention: float | None = None) -> None:
        self.enabled = enabled
        if retention is not None:
            if not 0 < retention <= 1:
                raise ValueError("retention must lie in (0, 1]")
            self.retention = float(retention)

    def forward(self, x: Tensor) -> Tensor:
        self._current_input = x
        try:
            return self.original(x)
        finally:
            self._current_input = None

    def close(self) -> None:
        if self._norm_hook is not None:
            self._norm_hook.remove()
            self._norm_hook = None
        if (self._accelerate_old_forward is not None
                and self.original.down_proj._old_forward is self._accelerate_interceptor):
            self.original.down_proj._old_forward = self._accelerate_old_forward
