"""Intermediate-dimension sharding emulated on one GPU: the P partials sum to the full layer."""
from __future__ import annotations

import pytest
import torch

from oracle import ffn as offn
import qcc_b200.workloads as workloads
from qcc_b200.runtime import IndexedSparseFFN
from qcc_b200.runtime.packing import PackedFFNWeights
from qcc_b200.runtime.selector import select_topk
from qcc_b200.runtime.sharded import ShardedIndexedFFN, shard_range

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_partials_sum_to_full_layer(world):
    layer = workloads.decode_layer(hidden=1024, intermediate=4096, device="cuda", seed=3)
    k = workloads.retention_k(4096, 0.25)
    ids = workloads.decode_ids(4096, k, token=2).cuda()
    x = workloads.decode_x(hidden=1024).cuda()
    full = IndexedSparseFFN(PackedFFNWeights(layer.packed, 1024, 4096))(x, ids, out_dtype=torch.float32)
    total = torch.zeros_like(full)
    for rank in range(world):
        b, e = shard_range(4096, world, rank)
        shard = ShardedIndexedFFN(PackedFFNWeights(layer.packed[b:e], 1024, e - b, b, 4096))
        total += shard.partial(x, ids)
    assert offn.rel_l2(total.double().cpu().numpy(), full.double().cpu().numpy()) <= 1e-5
    # The single-rank path (no process group) returns the cast full result.
    whole = ShardedIndexedFFN(PackedFFNWeights(layer.packed, 1024, 4096, 0, 4096))(x, ids)
    assert offn.rel_l2(whole.double().cpu().numpy(), full.double().cpu().numpy()) <= 1e-2


def test_per_token_rows_through_shards():
    layer = workloads.decode_layer(hidden=512, intermediate=2048, device="cuda", seed=4)
    scores = workloads.selector_scores(5, intermediate=2048, seed=9)
    rows = select_topk(scores.cuda(), 410)
    x = workloads.decode_x(batch=5, hidden=512).cuda()
    total = None
    for rank in range(4):
        b, e = shard_range(2048, 4, rank)
        part = ShardedIndexedFFN(PackedFFNWeights(layer.packed[b:e], 512, e - b, b, 2048)).partial(x, rows)
        total = part if total is None else total + part
    gate, up, down = layer.gate().cpu(), layer.up().cpu(), layer.down().cpu()
    for t in range(5):
        expected = offn.sparse_ffn_f64(x[t:t + 1].cpu(), rows[t].cpu(), gate, up, down)
        assert offn.rel_l2(total[t:t + 1].double().cpu().numpy(), expected) <= 1e-4
