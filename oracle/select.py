"""CPU restatement of top-K selection with the fixed tie rule (test infrastructure only).

The reference calls ``torch.topk(scores, k, sorted=False)`` (runtime/selector.py:24,
end_to_end/oracle_sparse_mlp.py:75) whose tie order is unspecified; the rule
checked here is ``sort(scores, descending, stable)[:k]`` then ascending: ties
go to the lower index, -0.0 == +0.0, NaN ranks largest.  Integer work, so the
GPU selector must match it bit for bit.
"""
from __future__ import annotations

import numpy as np


def score_keys(scores: np.ndarray) -> np.ndarray:
    """Order-preserving uint32 keys: larger score -> larger key; NaN -> max; -0 == +0."""
    f = np.ascontiguousarray(scores, dtype=np.float32)
    u = f.view(np.uint32).copy()
    u[(u & 0x7FFFFFFF) == 0] = 0
    neg = (u & 0x80000000) != 0
    keys = np.where(neg, ~u, u | np.uint32(0x80000000)).astype(np.uint32)
    keys[np.isnan(f)] = np.uint32(0xFFFFFFFF)
    return keys


def topk_ids(scores: np.ndarray, k: int) -> np.ndarray:
    """[B, N] -> [B, k] ascending int32 ids of the k largest (ties: lower index)."""
    scores = np.atleast_2d(np.asarray(scores, dtype=np.float32))
    keys = score_keys(scores).astype(np.int64)
    order = np.argsort(-keys, axis=-1, kind="stable")[:, :k]
    return np.sort(order, axis=-1).astype(np.int32)


def block_topk_indices(scores: np.ndarray, k: int, block_size: int) -> np.ndarray:
    """oracle/importance.py:26-35: complete blocks by summed score, expanded and sorted.

    Block order among equal sums follows the same lower-index tie rule.
    """
    scores = np.atleast_2d(np.asarray(scores, dtype=np.float32))
    n = scores.shape[-1]
    padded = (n + block_size - 1) // block_size * block_size
    block_scores = np.pad(scores, ((0, 0), (0, padded - n))).reshape(scores.shape[0], -1, block_size).sum(-1)
    blocks = max(1, min(block_scores.shape[-1], (k + block_size - 1) // block_size))
    chosen = topk_ids(block_scores, blocks).astype(np.int64)
    idx = (chosen[..., None] * block_size + np.arange(block_size)).reshape(scores.shape[0], -1)
    idx = np.where(idx >= n, n, idx)
    return np.sort(idx, axis=-1)[:, :min(blocks * block_size, n)]


def union_with_mask(rows: np.ndarray, begin: int, end: int):
    """Sorted distinct ids of all rows inside [begin, end), rebased, with token bits."""
    rows = np.atleast_2d(rows)
    bits = {}
    for b, row in enumerate(rows):
        for i in row.tolist():
            if begin <= i < end:
                bits[i - begin] = bits.get(i - begin, 0) | (1 << b)
    ids = np.array(sorted(bits), dtype=np.int32)
    mask = np.array([bits[i] for i in ids.tolist()], dtype=np.uint8)
    return ids, mask
