"""x-only oracle sparse MLP for real models, selecting on the GPU in one launch per call.

Interface of reference end_to_end/oracle_sparse_mlp.py:35-98: ``OracleSparseMLP(original,
layer_idx, retention=1.0, telemetry=None, norm_chunk_columns=256)`` wrapping a gated MLP
(``gate_proj`` / ``up_proj`` / ``down_proj`` / ``act_fn``), ``forward(x)`` only,
``set_mode(enabled, retention)``, ``last_selected_indices``, ``down_column_norms``,
``norm_computation_count``, ``norm_preparation_log``, ``close()``; and
``compute_down_column_norms_chunked(weight, chunk_columns)``.

How it works here:

* The wrapper always runs the original module, so a model's own hooks (Accelerate's
  weight materialisation included) stay in charge of gate, up and down.  A tap on
  ``down_proj`` (:class:`DownProjectionTap`) sees the activation a = act(gate x) * up x
  on its way in.
* In sparse mode the tap hands a to one ``qcc_activation_topk`` launch: per row the
  score |a| * ||D[:, j]||_2 (fp32, one rounding), the K = ceil(retention * N) best
  neurons with ties to the lower index, and the masked activation -- a on the selected
  neurons, 0 elsewhere -- written in the same pass.  ``down_proj`` then runs on the
  masked activation.  The reference needs abs, a cast, a multiply, ``torch.topk``,
  ``zeros_like``, ``gather`` and ``scatter_`` for the same step.
* The down-column norms are prepared lazily, on the first sparse call, by one pass of
  ``qcc_column_norms`` over the weight on its own device (fp64 accumulation, no fp32
  copy of the weight); host weights go through fp32 column chunks of
  ``norm_chunk_columns``.

The selected set is the reference's whenever the K-th and (K+1)-th scores differ (the
reference leaves ties to ``torch.topk``).  ``last_selected_indices`` is int64 [..., K],
ascending.  Sparse mode on a host tensor raises (there is no CPU fallback).
"""
from __future__ import annotations

import math
from typing import Callable

import torch
from torch import Tensor, nn

from .. import _lib
from ..runtime.selector import activation_topk


@torch.no_grad()
def compute_down_column_norms_chunked(weight: Tensor, chunk_columns: int = 256) -> Tensor:
    """fp32 ||W[:, j]||_2 of every column of the down projection W [hidden, N], on W's device.

    CUDA weights: one ``qcc_column_norms`` pass.  Host weights: at most
    ``hidden x chunk_columns`` values are widened to fp32 at a time.
    """
    if weight.ndim != 2:
        raise ValueError("down projection weight must be a matrix")
    if chunk_columns <= 0:
        raise ValueError("chunk_columns must be positive")
    if weight.device.type == "meta":
        raise RuntimeError("down projection is still meta; Accelerate did not materialize it before the pre-hook")
    rows, cols = weight.shape
    out = torch.empty(cols, dtype=torch.float32, device=weight.device)
    if weight.is_cuda and weight.dtype in _lib.TORCH_DTYPES:
        w = weight.detach()
        if w.stride(1) != 1:
            w = w.contiguous()
        lib = _lib.library()
        with torch.cuda.device(w.device):
            _lib.check(lib.qcc_column_norms(w.data_ptr(), w.stride(0), rows, cols, _lib.dtype_code(w.dtype),
                                            out.data_ptr(), _lib.stream_handle(w.device)), "qcc_column_norms")
        return out
    for lo in range(0, cols, chunk_columns):
        hi = min(cols, lo + chunk_columns)
        out[lo:hi] = weight.detach()[:, lo:hi].to(torch.float32).square().sum(dim=0).sqrt()
    return out


def telemetry_metrics(dense: Tensor, sparse: Tensor, eps: float = 1e-12) -> dict[str, Tensor]:
    """Per-row agreement of the dense and sparse down outputs [rows, hidden].

    The keys are the ones the reference's telemetry consumers read (evaluation/metrics.py:
    cosine_similarity, relative_l2, mse, max_absolute_error); identical rows count as cosine 1.
    """
    d = dense.float()
    s = sparse.float()
    err = d - s
    d_norm = d.norm(dim=-1)
    s_norm = s.norm(dim=-1)
    cosine = torch.clamp((d * s).sum(-1) / torch.clamp(d_norm * s_norm, min=eps), -1.0, 1.0)
    cosine = torch.where(err.eq(0).all(-1), torch.ones_like(cosine), cosine)
    return {"cosine_similarity": cosine, "relative_l2": err.norm(dim=-1) / (d_norm + eps),
            "mse": err.pow(2).mean(-1), "max_absolute_error": err.abs().amax(-1)}


class DownProjectionTap:
    """Lets a handler rewrite the activation entering a ``down_proj`` module, removably.

    Accelerate-dispatched modules (``_hf_hook`` + ``_old_forward``) materialise their
    weight inside the rewritten ``forward`` after ordinary pre-hooks have run, so for them
    the inner ``_old_forward`` is wrapped; every other module gets a forward pre-hook.
    ``handler(module, activation)`` returns a replacement activation or None.
    """

    def __init__(self, module: nn.Module, handler: Callable[[nn.Module, Tensor], Tensor | None]):
        self.module = module
        self._handler = handler
        self._hook = None
        self._inner = None
        if hasattr(module, "_hf_hook") and hasattr(module, "_old_forward"):
            self._inner = module._old_forward

            def wrapped(activation, *rest, **kwargs):
                swapped = handler(module, activation)
                return self._inner(activation if swapped is None else swapped, *rest, **kwargs)

            self._wrapped = wrapped
            module._old_forward = wrapped
        else:
            def pre_hook(mod, args):
                swapped = handler(mod, args[0])
                return None if swapped is None else (swapped, *args[1:])

            self._hook = module.register_forward_pre_hook(pre_hook)

    def release(self) -> None:
        if self._hook is not None:
            self._hook.remove()
            self._hook = None
        if self._inner is not None:
            if getattr(self.module, "_old_forward", None) is self._wrapped:
                self.module._old_forward = self._inner
            self._inner = None


class OracleSparseMLP(nn.Module):
    """Keeps, per token, the neurons of a gated MLP that matter most for its own input."""

    actual_oracle_executes_dense_gate_up = True  # gate and up run dense: the selection needs every activation
    runtime_speedup_claimed = False              # an evaluation tool: the model still stores and reads every weight

    def __init__(self, original: nn.Module, layer_idx: int, retention: float = 1.0,
                 telemetry: Callable[[int, dict[str, Tensor]], None] | None = None,
                 norm_chunk_columns: int = 256):
        super().__init__()
        if norm_chunk_columns <= 0:
            raise ValueError("norm_chunk_columns must be positive")
        self.original = original
        self.layer_idx = layer_idx
        self.retention = float(retention)
        self.telemetry = telemetry
        self.norm_chunk_columns = norm_chunk_columns
        self.enabled = False
        self.norm_computation_count = 0
        self.norm_preparation_log: dict | None = None
        self.last_selected_indices: Tensor | None = None
        self._x: Tensor | None = None
        self.register_buffer("down_column_norms", None, persistent=False)
        self._tap = DownProjectionTap(original.down_proj, self._on_down_input)

    @property
    def intermediate_size(self) -> int:
        return int(self.original.down_proj.weight.shape[1])

    def set_mode(self, enabled: bool, retention: float | None = None) -> None:
        if retention is not None and not 0 < retention <= 1:
            raise ValueError("retention must lie in (0, 1]")
        self.enabled = bool(enabled)
        if retention is not None:
            self.retention = float(retention)

    def forward(self, x: Tensor) -> Tensor:
        self._x = x
        try:
            return self.original(x)
        finally:
            self._x = None

    def close(self) -> None:
        self._tap.release()

    # -- the sparse step -------------------------------------------------------------

    def _prepare_norms(self, weight: Tensor) -> Tensor:
        if self.down_column_norms is None:
            norms = compute_down_column_norms_chunked(weight, self.norm_chunk_columns)
            self.down_column_norms = norms
            self.norm_computation_count += 1
            self.norm_preparation_log = {
                "layer": self.layer_idx, "weight_shape": tuple(weight.shape), "weight_dtype": str(weight.dtype),
                "device": str(weight.device),
                "method": "qcc_column_norms (one pass, fp64 sums)" if weight.is_cuda
                else f"host fp32 chunks of {self.norm_chunk_columns} columns",
                "norm_bytes": norms.numel() * norms.element_size()}
        return self.down_column_norms

    def _on_down_input(self, module: nn.Module, activation: Tensor) -> Tensor | None:
        if not self.enabled or self.retention >= 1.0:
            return None  # dense: no norms, no selection
        if not activation.is_cuda:
            raise RuntimeError("OracleSparseMLP sparse mode runs on CUDA tensors only (no CPU fallback)")
        n = self.intermediate_size
        k = min(n, max(1, math.ceil(self.retention * n)))
        norms = self._prepare_norms(module.weight).to(activation.device)
        rows = activation.detach().reshape(-1, n)
        ids, sparse_rows = activation_topk(rows, k, norms, masked=True)
        self.last_selected_indices = ids.long().reshape(*activation.shape[:-1], k)
        sparse = sparse_rows.reshape(activation.shape)
        if self.telemetry is not None:
            self._report(module, activation, sparse)
        return sparse

    def _report(self, module: nn.Module, activation: Tensor, sparse: Tensor) -> None:
        weight, bias = module.weight, getattr(module, "bias", None)
        dense_out = nn.functional.linear(activation, weight, bias).flatten(0, -2)
        sparse_out = nn.functional.linear(sparse, weight, bias).flatten(0, -2)
        stats = telemetry_metrics(dense_out, sparse_out)
        residual = self._x.float().flatten(0, -2).norm(dim=-1).clamp_min(1e-12)
        stats["ffn_over_residual"] = dense_out.float().norm(dim=-1) / residual
        stats["ffn_error_over_residual"] = (dense_out - sparse_out).float().norm(dim=-1) / residual
        self.telemetry(self.layer_idx, stats)
