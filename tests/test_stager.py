"""Host-offload stager: cache policy against the reference LRU, the layer against the oracle on the GPU."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_json
from oracle import ffn as offn
from oracle import lru as olru
import qcc_b200.workloads as workloads


def test_slot_cache_with_no_hot_set_is_the_reference_lru():
    data = load_json("lru_cases.json")
    for case in data["cases"].values():
        cache = olru.SlotCache(data["neuron_count"], [], case["capacity_neurons"])
        for t, (row, expected) in enumerate(zip(data["masks"], case["events"])):
            got = cache.step(sorted(row), t)
            assert (got["hits"], got["misses"], got["evicted"]) == (expected["hits"], expected["misses"],
                                                                     expected["evicted"])


def test_slot_cache_matches_lru_events_on_a_long_sequence():
    seqs = workloads.offload_token_ids(300, 40, torch.tensor([], dtype=torch.long), tokens=30, seed=3)
    masks = [s.tolist() for s in seqs]
    cache = olru.SlotCache(300, [], 64)
    events = olru.lru_events(masks, 64)
    for t, row in enumerate(masks):
        got = cache.step(row, t)
        assert (got["hits"], got["misses"], got["evicted"]) == (events[t]["hits"], events[t]["misses"],
                                                                 events[t]["evicted"])


def test_offload_workload_shape():
    hot = workloads.offload_hot_set(17408)
    assert hot.numel() == 4352
    k = workloads.retention_k(17408, 0.1)
    seqs = workloads.offload_token_ids(17408, k, hot, tokens=4)
    is_hot = torch.zeros(17408, dtype=torch.bool)
    is_hot[hot] = True
    first = seqs[0].long()
    assert first.numel() == k == 1741 and bool((first[1:] > first[:-1]).all())
    assert int(is_hot[first].sum()) == round(0.8 * k)
    overlap = np.intersect1d(seqs[0].numpy(), seqs[1].numpy()).size
    assert overlap >= round(0.5 * k)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_offload_layer_matches_oracle_and_policy(dtype):
    from qcc_b200.runtime.stager import HostOffloadLayer

    hidden, n, k, tokens = 256, 1200, 120, 12
    layer = workloads.decode_layer(hidden=hidden, intermediate=n, dtype=dtype, device="cpu", seed=9)
    hot = workloads.offload_hot_set(n, seed=4)
    seqs = workloads.offload_token_ids(n, k, hot, tokens=tokens, seed=5)
    capacity = 64
    stager = HostOffloadLayer(layer.packed, hidden, hot, capacity=capacity, max_k=k, device="cuda")
    cache = olru.SlotCache(n, hot.tolist(), capacity)
    x = workloads.decode_x(hidden=hidden, dtype=dtype).cuda()
    gate, up, down = layer.gate(), layer.up(), layer.down()
    for t, ids in enumerate(seqs):
        y = stager(x, ids.cuda())
        expect = cache.step(ids.tolist(), t)
        stats = stager.stats()
        assert stats["overflow"] == 0
        assert (stats["cache_hits"], stats["misses"], stats["evicted"], stats["hot_hits"]) == (
            expect["hits"], expect["misses"], expect["evicted"], expect["hot_hits"])
        assert stager.resident_ids[:stats["resident"]].tolist() == expect["resident"]
        assert stager.miss_slot[:stats["misses"]].tolist() == expect["miss_slots"]
        assert stager.slot_of.tolist() == cache.slot_of
        reference = offn.sparse_ffn_f64(x.cpu(), ids, gate, up, down)
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        assert offn.rel_l2(y.double().cpu().numpy(), reference) <= tol


@pytest.mark.gpu
def test_offload_capacity_overflow_is_reported():
    from qcc_b200.runtime.stager import HostOffloadLayer

    hidden, n = 64, 400
    layer = workloads.decode_layer(hidden=hidden, intermediate=n, device="cpu", seed=2)
    hot = torch.arange(0, 100)
    stager = HostOffloadLayer(layer.packed, hidden, hot, capacity=8, max_k=64, device="cuda")
    ids = torch.arange(100, 120, dtype=torch.int32).cuda()  # 20 cold ids > 8 slots
    stager(workloads.decode_x(hidden=hidden).cuda(), ids)
    stats = stager.stats()
    assert stats["overflow"] == 1 and stats["misses"] == 8


@pytest.mark.gpu
def test_decode_accumulate_adds_a_partial_result():
    from qcc_b200.runtime import IndexedSparseFFN
    from qcc_b200.runtime.packing import PackedFFNWeights

    layer = workloads.decode_layer(hidden=512, intermediate=800, device="cuda", seed=6)
    engine = IndexedSparseFFN(PackedFFNWeights(layer.packed, 512, 800))
    x = workloads.decode_x(hidden=512).cuda()
    ids = workloads.decode_ids(800, 200, token=3).cuda()
    first = engine(x, ids[:120], out_dtype=torch.float32)
    both = engine(x, ids[120:], accumulate=first, out_dtype=torch.float32)
    whole = engine(x, ids, out_dtype=torch.float32)
    assert offn.rel_l2(both.double().cpu().numpy(), whole.double().cpu().numpy()) <= 1e-5


@pytest.mark.gpu
def test_gather_refuses_pageable_host_memory():
    from qcc_b200 import _lib

    lib = _lib.library()
    store = torch.zeros(64, dtype=torch.uint8)  # ordinary (pageable) host memory
    idx = torch.zeros(1, dtype=torch.int32, device="cuda")
    dst = torch.zeros(64, dtype=torch.uint8, device="cuda")
    status = lib.qcc_gather_records(store.data_ptr(), 64, idx.data_ptr(), idx.data_ptr(), None, 1, dst.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    assert status == _lib.ERR_INVALID_ARGUMENT


@pytest.mark.gpu
def test_offload_full_size_eight_layers():
    """The low-VRAM offload configuration at full size: 8 layers of hidden 5120 x N 17408 (bf16),
    a quarter of each layer's records hot in HBM, K/N = 0.1 per token (80 % from the hot set, half
    reused from the previous token), 2048 cache slots.  The cache policy is checked against the
    oracle's slot cache at every step of every layer, y against the float64 oracle at the first
    and last token of every layer."""
    from qcc_b200.runtime.stager import HostOffloadLayer

    hidden, n, layers, tokens, capacity = 5120, 17408, 8, 6, 2048
    k = workloads.retention_k(n, 0.1)
    x = workloads.decode_x().cuda()
    for l in range(layers):
        packed = workloads.decode_layer(device="cuda", seed=100 + l).packed.cpu()
        hot = workloads.offload_hot_set(n, seed=11 + l)
        seqs = workloads.offload_token_ids(n, k, hot, tokens, seed=12 + l)
        stager = HostOffloadLayer(packed, hidden, hot, capacity=capacity, max_k=k, device="cuda")
        cache = olru.SlotCache(n, hot.tolist(), capacity)
        gate, up, down = packed[:, :hidden], packed[:, hidden:2 * hidden], packed[:, 2 * hidden:].t()
        for t, ids in enumerate(seqs):
            y = stager(x, ids.cuda())
            expect = cache.step(ids.tolist(), t)
            stats = stager.stats()
            assert stats["overflow"] == 0
            assert (stats["cache_hits"], stats["misses"], stats["evicted"], stats["hot_hits"]) == (
                expect["hits"], expect["misses"], expect["evicted"], expect["hot_hits"]), (l, t)
            assert stager.miss_slot[:stats["misses"]].tolist() == expect["miss_slots"]
            if t in (0, tokens - 1):
                assert stager.slot_of.tolist() == cache.slot_of
                reference = offn.sparse_ffn_f64(x.cpu(), ids, gate, up, down)
                assert offn.rel_l2(y.double().cpu().numpy(), reference) <= 1e-2, (l, t)
        del stager, packed
        torch.cuda.empty_cache()
