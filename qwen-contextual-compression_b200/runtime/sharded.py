"""Intermediate-dimension sharding of one FFN layer over GPUs (one process per GPU).

Rank r of P owns the contiguous records [r*N//P, (r+1)*N//P).  Every rank
holds the same global selected ids (the selector is deterministic and
replicated), keeps the ones inside its range, rebased (qcc_build_union, one
small launch), runs the fused kernel with an fp32 partial output, and the P
partials are summed with an NCCL all-reduce on the compute stream before a
cast to the weight dtype.  Only y (hidden fp32 values per token, 20 KB at
hidden 5120) crosses NVLink.  The reference has no distributed path
(integration/freetoken_qcc/low_vram/adapter.py:106-107 refuses TP != 1).
"""
from __future__ import annotations

import torch

from .. import _lib
from .engine import IndexedSparseFFN
from .packing import PackedFFNWeights
from .selector import build_union


def shard_range(intermediate: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous record range of `rank` among `world` shards."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return intermediate * rank // world, intermediate * (rank + 1) // world


class ShardedIndexedFFN:
    """One rank's slice of an indexed sparse FFN layer plus the cross-rank sum."""

    def __init__(self, weights: PackedFFNWeights, group=None):
        self.weights = weights
        self.engine = IndexedSparseFFN(weights)
        self.group = group
        self.begin = weights.record_offset
        self.end = weights.record_offset + weights.n_records

    def partial(self, x: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        """fp32 partial y of this rank's records; ids are global ([K] shared or [B, K] per token)."""
        rows = ids if ids.ndim == 2 else ids.unsqueeze(0)
        if rows.dtype != torch.int32:
            rows = rows.to(torch.int32)
        rows = rows.contiguous()
        local, mask, count = build_union(rows, self.begin, self.end)
        per_token = ids.ndim == 2
        x2 = x if x.ndim == 2 else x.unsqueeze(0)
        return self.engine(x2, local, token_mask=mask if per_token else None, n_ids_dev=count,
                           out_dtype=torch.float32)

    def __call__(self, x: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        return self.forward(x, ids)

    def forward(self, x: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        y32 = self.partial(x, ids)
        if self.group is not None:
            torch.distributed.all_reduce(y32, group=self.group)
        out = torch.empty(y32.shape, dtype=self.weights.dtype, device=y32.device)
        lib = _lib.library()
        _lib.check(lib.qcc_cast_f32(y32.data_ptr(), out.data_ptr(), y32.numel(), _lib.dtype_code(out.dtype),
                                    _lib.stream_handle(y32.device)), "qcc_cast_f32")
        return out if x.ndim == 2 else out.squeeze(0)

    def close(self) -> None:
        self.engine = None
