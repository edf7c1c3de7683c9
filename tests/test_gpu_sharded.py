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


@pytest.mark.parametrize("ids_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("batch", [1, 3])
def test_in_kernel_shard_range_matches_union(ids_dtype, batch):
    """Global ascending ids + id_range == rebased union ids, bit for bit, per shard."""
    hidden, n, world = 1024, 4096, 4
    layer = workloads.decode_layer(hidden=hidden, intermediate=n, device="cuda", seed=6)
    k = workloads.retention_k(n, 0.25)
    ids = workloads.decode_ids(n, k, token=3).cuda()
    x = workloads.decode_x(batch=batch, hidden=hidden).cuda()
    gate, up, down = layer.gate().cpu(), layer.up().cpu(), layer.down().cpu()
    total = torch.zeros((batch, hidden), dtype=torch.float64)
    for rank in range(world):
        b, e = shard_range(n, world, rank)
        engine = IndexedSparseFFN(PackedFFNWeights(layer.packed[b:e], hidden, e - b, b, n))
        ranged = engine(x, ids.to(ids_dtype), id_range=(b, e), out_dtype=torch.float32)
        local = (ids[(ids >= b) & (ids < e)] - b).to(torch.int32)
        # A device count keeps the grid at one CTA per SM, as in the ranged call.
        count = torch.tensor([local.numel()], dtype=torch.int32, device="cuda")
        rebased = engine(x, local, n_ids_dev=count, out_dtype=torch.float32)
        assert torch.equal(ranged, rebased)
        engine.check()
        total += ranged.double().cpu()
    for t in range(batch):
        expected = offn.sparse_ffn_f64(x[t:t + 1].cpu(), ids.cpu(), gate, up, down)
        assert offn.rel_l2(total[t:t + 1].numpy(), expected) <= 1e-4


def test_in_kernel_shard_range_edges():
    """Empty shard, shard outside every id, and a device-side id count."""
    hidden, n = 512, 2048
    layer = workloads.decode_layer(hidden=hidden, intermediate=n, device="cuda", seed=7)
    x = workloads.decode_x(hidden=hidden).cuda()
    ids = torch.arange(0, 1024, 3, dtype=torch.int32, device="cuda")  # all below 1024
    hi = IndexedSparseFFN(PackedFFNWeights(layer.packed[1024:], hidden, n - 1024, 1024, n))
    y = hi(x, ids, id_range=(1024, n), out_dtype=torch.float32)
    assert torch.count_nonzero(y) == 0
    empty = IndexedSparseFFN(PackedFFNWeights(layer.packed[:0], hidden, 0, 0, n))
    assert torch.count_nonzero(empty(x, ids, id_range=(0, 0), out_dtype=torch.float32)) == 0
    lo = IndexedSparseFFN(PackedFFNWeights(layer.packed[:1024], hidden, 1024, 0, n))
    count = torch.tensor([100], dtype=torch.int32, device="cuda")
    ranged = lo(x, ids, id_range=(0, 1024), n_ids_dev=count, out_dtype=torch.float32)
    plain = lo(x, ids, n_ids_dev=count, out_dtype=torch.float32)
    assert torch.equal(ranged, plain)
    for e in (hi, empty, lo):
        e.check()
