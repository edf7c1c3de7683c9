"""Deterministic top-K selection and per-token unions on the GPU.

The reference selects with ``torch.topk(scores, k, sorted=False)``
(runtime/selector.py:24, runtime/cuda_selector.py:40,
end_to_end/oracle_sparse_mlp.py:75), whose order -- and whose choice among
tied scores -- is unspecified.  :func:`select_topk` returns the k largest
scores per row as ascending unique int32 indices with ties broken by lower
index, -0.0 equal to +0.0 and NaN ranked largest: exactly
``sort(scores, descending=True, stable=True)[:k]`` sorted ascending, which
is always one of the answers torch.topk may give.
"""
from __future__ import annotations

import math

import torch

from .. import _lib


def retention_count(width: int, retention: float) -> int:
    """K = max(1, ceil(width * retention)) (predictor/candidate_reranker.py:9-12)."""
    if not 0 < retention <= 1:
        raise ValueError("retention must be in (0, 1]")
    return max(1, math.ceil(width * retention))


def select_topk(scores: torch.Tensor, k: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """[B, N] or [N] fp32 scores -> [B, k] (or [k]) ascending int32 indices."""
    squeeze = scores.ndim == 1
    if squeeze:
        scores = scores.unsqueeze(0)
    if scores.ndim != 2:
        raise ValueError("scores must be [batch, n] or [n]")
    if scores.dtype != torch.float32:
        raise TypeError("scores must be float32")
    device = _lib.require_cuda(scores)
    if scores.stride(1) != 1:
        scores = scores.contiguous()
    batch, n = scores.shape
    if not 0 <= k <= n:
        raise ValueError(f"k must be in [0, {n}]")
    if out is None:
        out = torch.empty((batch, k), dtype=torch.int32, device=device)
    elif out.shape != (batch, k) or out.dtype != torch.int32 or out.stride(1) != 1:
        raise ValueError("out must be a row-contiguous int32 [batch, k] tensor")
    lib = _lib.library()
    status = lib.qcc_select_topk(scores.data_ptr(), scores.stride(0), batch, n, k, out.data_ptr(), out.stride(0),
                                 _lib.stream_handle(device))
    _lib.check(status, "qcc_select_topk")
    return out.squeeze(0) if squeeze else out


def activation_topk(act: torch.Tensor, k: int, col_weights: torch.Tensor | None = None, *, masked: bool = False,
                    out: torch.Tensor | None = None):
    """Scores made from an activation and their top k, in one launch (``qcc_activation_topk``).

    act [R, N] (or [N]) in bf16 / fp16 / fp32; score = |a| * col_weights
    (fp32 [N]) or |a|.  Returns ascending int32 ids [R, k] -- and, with
    ``masked=True``, also act with every unselected entry set to 0.
    """
    squeeze = act.ndim == 1
    if squeeze:
        act = act.unsqueeze(0)
    if act.ndim != 2:
        raise ValueError("act must be [rows, n] or [n]")
    device = _lib.require_cuda(act, col_weights, out)
    code = _lib.dtype_code(act.dtype)
    if act.stride(1) != 1:
        act = act.contiguous()
    rows, n = act.shape
    if not 0 <= k <= n:
        raise ValueError(f"k must be in [0, {n}]")
    if col_weights is not None and (col_weights.dtype != torch.float32 or col_weights.numel() != n
                                    or not col_weights.is_contiguous()):
        raise ValueError("col_weights must be a contiguous float32 tensor with one weight per column")
    if out is None:
        out = torch.empty((rows, k), dtype=torch.int32, device=device)
    elif out.shape != (rows, k) or out.dtype != torch.int32 or out.stride(1) != 1:
        raise ValueError("out must be a row-contiguous int32 [rows, k] tensor")
    sparse = torch.empty_like(act) if masked else None
    lib = _lib.library()
    status = lib.qcc_activation_topk(act.data_ptr(), act.stride(0), code, rows, n, _lib.ptr(col_weights), k,
                                     out.data_ptr(), out.stride(0), _lib.ptr(sparse),
                                     sparse.stride(0) if sparse is not None else 0, _lib.stream_handle(device))
    _lib.check(status, "qcc_activation_topk")
    if squeeze:
        out = out.squeeze(0)
        sparse = None if sparse is None else sparse.squeeze(0)
    return (out, sparse) if masked else out


def block_topk(scores: torch.Tensor, k: int, block: int, *, with_sums: bool = False):
    """Block top-K of fp32 score rows [R, N] (reference oracle/importance.py:26-35).

    Returns ascending int32 block ids [R, kb], kb = max(1, min(ceil(N / block),
    ceil(k / block))); block j covers neurons [j * block, min(N, (j+1) * block)).
    ``with_sums=True`` also returns the fp32 block sums [R, ceil(N / block)].
    """
    squeeze = scores.ndim == 1
    if squeeze:
        scores = scores.unsqueeze(0)
    if scores.ndim != 2 or scores.dtype != torch.float32:
        raise ValueError("scores must be float32 [rows, n] or [n]")
    if block <= 0:
        raise ValueError("block_size must be positive")
    device = _lib.require_cuda(scores)
    if scores.stride(1) != 1:
        scores = scores.contiguous()
    rows, n = scores.shape
    if not 1 <= k <= n:
        raise ValueError(f"k must be in [1, {n}]")
    n_blocks = (n + block - 1) // block
    kb = max(1, min(n_blocks, (k + block - 1) // block))
    ids = torch.empty((rows, kb), dtype=torch.int32, device=device)
    sums = torch.empty((rows, n_blocks), dtype=torch.float32, device=device) if with_sums else None
    lib = _lib.library()
    _lib.check(lib.qcc_block_topk(scores.data_ptr(), scores.stride(0), rows, n, block, k, ids.data_ptr(), kb,
                                  _lib.ptr(sums), n_blocks, _lib.stream_handle(device)), "qcc_block_topk")
    if squeeze:
        ids = ids[0]
        sums = None if sums is None else sums[0]
    return (ids, sums) if with_sums else ids


def tile_block_union(block_ids: torch.Tensor, n_blocks: int, tile_rows: int = 128):
    """Per tile of ``tile_rows`` rows, the ascending union of the rows' block ids.

    Returns (flat int32 [capacity], offsets int32 [tiles + 1]) on the device --
    the per-tile block lists ``BlockSparsePrefill`` takes.
    """
    if block_ids.ndim != 2 or block_ids.dtype != torch.int32 or block_ids.stride(1) != 1:
        raise ValueError("block_ids must be a row-contiguous int32 [rows, kb] tensor")
    device = _lib.require_cuda(block_ids)
    rows, kb = block_ids.shape
    tiles = (rows + tile_rows - 1) // tile_rows
    flat = torch.empty(max(1, tiles * n_blocks), dtype=torch.int32, device=device)
    offsets = torch.empty(tiles + 1, dtype=torch.int32, device=device)
    lib = _lib.library()
    _lib.check(lib.qcc_tile_block_union(block_ids.data_ptr(), block_ids.stride(0), rows, kb, tile_rows, n_blocks,
                                        flat.data_ptr(), offsets.data_ptr(), None, _lib.stream_handle(device)),
               "qcc_tile_block_union")
    return flat, offsets


def build_union(ids: torch.Tensor, id_begin: int = 0, id_end: int | None = None, capacity: int | None = None):
    """Union of per-token sorted id rows [B, k] (B <= 8) restricted to [id_begin, id_end).

    Returns (union_ids int32 [capacity], token_mask uint8 [capacity], count
    int32 [1] on the device).  Entries past ``count`` are undefined.  Ids are
    rebased to id_begin (local to an intermediate-dimension shard).
    """
    if ids.ndim == 1:
        ids = ids.unsqueeze(0)
    if ids.ndim != 2 or ids.dtype != torch.int32 or ids.stride(1) != 1:
        raise ValueError("ids must be a row-contiguous int32 [batch, k] tensor")
    device = _lib.require_cuda(ids)
    batch, k = ids.shape
    if not 1 <= batch <= 8:
        raise ValueError("build_union handles 1..8 token rows")
    if id_end is None:
        id_end = int(ids.max().item()) + 1 if ids.numel() else id_begin
    width = id_end - id_begin
    if width < 0:
        raise ValueError("id_end must be >= id_begin")
    cap = min(width, batch * k) if capacity is None else capacity
    if cap < min(width, batch * k):
        raise ValueError("capacity below min(id_end - id_begin, batch * k)")
    union_ids = torch.empty(max(cap, 1), dtype=torch.int32, device=device)
    token_mask = torch.empty(max(cap, 1), dtype=torch.uint8, device=device)
    count = torch.empty(1, dtype=torch.int32, device=device)
    lib = _lib.library()
    status = lib.qcc_build_union(ids.data_ptr(), ids.stride(0), batch, k, id_begin, id_end, union_ids.data_ptr(),
                                 token_mask.data_ptr(), count.data_ptr(), _lib.stream_handle(device))
    _lib.check(status, "qcc_build_union")
    return union_ids, token_mask, count


class TopKSelector:
    """x-independent part of reference runtime/selector.py:15-24: scores -> ids.

    The score producer (the learned predictor) is outside the hot path; this
    takes per-neuron scores and applies the retention, returning ascending
    int32 ids [B, K].
    """

    def __init__(self, intermediate: int, retention: float = 0.5):
        self.intermediate = intermediate
        self.retention = retention
        self.k = retention_count(intermediate, retention)

    def select(self, scores: torch.Tensor) -> torch.Tensor:
        if scores.shape[-1] != self.intermediate:
            raise ValueError(f"expected {self.intermediate} scores per row, got {scores.shape[-1]}")
        return select_topk(scores.float(), self.k)


def selected_set_comparison(reference: torch.Tensor, candidate: torch.Tensor, width: int) -> dict:
    """Set agreement of two [B, K] id lists (reference runtime/selector.py:51-52)."""
    ref = torch.zeros((len(reference), width), device=reference.device, dtype=torch.bool)
    ref.scatter_(-1, reference.long(), True)
    other = torch.zeros_like(ref).scatter_(-1, candidate.long().to(ref.device), True)
    intersection = (ref & other).sum(-1).float()
    changed = (ref ^ other).sum(-1).float()
    union = (ref | other).sum(-1).float().clamp_min(1)
    return {"set_equality_fraction": float((changed == 0).float().mean()),
            "jaccard": float((intersection / union).mean()),
            "mean_changed_neurons": float(changed.mean()),
            "p95_changed_neurons": float(changed.quantile(.95))}
