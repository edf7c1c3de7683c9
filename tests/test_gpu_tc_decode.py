"""Decode of 2-8 tokens on the tensor cores against the float64 oracle.

Two to eight tokens of bf16 / fp16 records whose hidden size is a multiple of
128 run the tensor-core kernel (records staged in groups of 16, the
activations split into a 16-bit high part and its remainder); these cases
cover odd token counts (padded to even), groups of 1-16 records, odd groups,
ids outside the records, the per-record activation output, the oracle-mode
passes and a full-size layer.  Tolerances: 1e-2 relative L2 for 16-bit
outputs, 1e-4 for fp32 outputs of 16-bit weights (the fp32 accumulation
order differs from the oracle's float64 sums).
"""
from __future__ import annotations

import pytest
import torch

from oracle import ffn as offn
import qcc_b200.workloads as workloads
from qcc_b200.runtime import IndexedSparseFFN, cuda_indexed_parts
from qcc_b200.runtime.oracle_mode import OracleModeFFN
from qcc_b200.runtime.packing import PackedFFNWeights, pack_neuron_major
from qcc_b200.runtime.selector import build_union, select_topk

pytestmark = pytest.mark.gpu


def _layer(h, n, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    gate = (torch.randn(n, h, generator=g) * 0.03).to(dtype)
    up = (torch.randn(n, h, generator=g) * 0.03).to(dtype)
    down = (torch.randn(h, n, generator=g) * 0.03).to(dtype)
    return gate, up, down


def _mask(n_ids, batch, seed):
    g = torch.Generator().manual_seed(seed)
    m = torch.randint(0, 256, (n_ids,), generator=g, dtype=torch.int64) & ((1 << batch) - 1)
    m[torch.arange(n_ids) % 5 == 0] = (1 << batch) - 1  # every token keeps some records
    return m.to(torch.uint8)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("batch", [2, 3, 4, 5, 6, 7, 8])
def test_batches_with_token_mask(batch, dtype):
    h, n = 1024, 3000
    gate, up, down = _layer(h, n, dtype, seed=batch)
    engine = IndexedSparseFFN(pack_neuron_major(gate.cuda(), up.cuda(), down.cuda()))
    assert engine.max_batch == 8
    # 2500 ids over 148 CTAs: runs of 16-17 records, one odd group per CTA.
    ids = torch.randperm(n, generator=torch.Generator().manual_seed(batch))[:2500].sort().values.int()
    mask = _mask(ids.numel(), batch, seed=batch)
    x = torch.randn(batch, h, generator=torch.Generator().manual_seed(100 + batch)).to(dtype)
    expected = offn.sparse_ffn_f64(x, ids, gate, up, down, token_mask=mask)
    y = engine(x.cuda(), ids.cuda(), token_mask=mask.cuda())
    assert y.dtype == dtype and offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-2
    y32 = engine(x.cuda(), ids.cuda(), token_mask=mask.cuda(), out_dtype=torch.float32)
    assert offn.rel_l2(y32.double().cpu().numpy(), expected) <= 1e-4
    engine.check()


@pytest.mark.parametrize("hidden,batch", [(8192, 6), (10240, 4), (3584, 8)])
def test_larger_hidden_sizes(hidden, batch):
    # y tiles of 1024 elements: 8 / 10 / 4 (the last one partial at 3584).
    n = 700
    gate, up, down = _layer(hidden, n, torch.bfloat16, seed=hidden)
    engine = IndexedSparseFFN(pack_neuron_major(gate.cuda(), up.cuda(), down.cuda()))
    assert engine.max_batch >= batch
    ids = torch.randperm(n, generator=torch.Generator().manual_seed(hidden))[:400].int()
    x = torch.randn(batch, hidden, generator=torch.Generator().manual_seed(5)).bfloat16()
    y = engine(x.cuda(), ids.cuda(), out_dtype=torch.float32)
    expected = offn.sparse_ffn_f64(x, ids, gate, up, down)
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-4


@pytest.mark.parametrize("n_ids", [1, 7, 150, 300, 4099])
def test_group_sizes_and_repeatability(n_ids):
    # 1-28 records per CTA: single records, odd groups, several full groups.
    h, n, batch = 2048, 5000, 4
    gate, up, down = _layer(h, n, torch.bfloat16, seed=n_ids)
    engine = IndexedSparseFFN(pack_neuron_major(gate.cuda(), up.cuda(), down.cuda()))
    ids = torch.randperm(n, generator=torch.Generator().manual_seed(n_ids))[:n_ids].int()
    x = torch.randn(batch, h, generator=torch.Generator().manual_seed(7)).bfloat16()
    y = engine(x.cuda(), ids.cuda(), out_dtype=torch.float32)
    expected = offn.sparse_ffn_f64(x, ids, gate, up, down)
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-4
    y2 = engine(x.cuda(), ids.cuda(), out_dtype=torch.float32)
    assert torch.equal(y, y2)  # fixed order of every sum: bit-reproducible


def test_ids_outside_the_records_are_flagged_and_skipped():
    h, n, batch = 1024, 400, 4
    gate, up, down = _layer(h, n, torch.bfloat16, seed=11)
    engine = IndexedSparseFFN(pack_neuron_major(gate.cuda(), up.cuda(), down.cuda()))
    bad = torch.tensor([3, 399, 400, -1, 17, 5000, 250], dtype=torch.int32)
    x = torch.randn(batch, h, generator=torch.Generator().manual_seed(12)).bfloat16()
    y = engine(x.cuda(), bad.cuda(), out_dtype=torch.float32)
    with pytest.raises(ValueError, match="range"):
        engine.check()
    good = torch.tensor([3, 399, 17, 250])
    expected = offn.sparse_ffn_f64(x, good, gate, up, down)
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-4


def test_empty_shard_at_four_tokens():
    # A layer slice with no records: every id is outside it, y is zero and the ids are flagged.
    layer = workloads.decode_layer(hidden=1024, intermediate=2048, device="cuda", seed=13)
    empty = IndexedSparseFFN(PackedFFNWeights(layer.packed[:0], 1024, 0, 0, 2048))
    x = workloads.decode_x(batch=4, hidden=1024).cuda()
    ids = torch.arange(0, 600, dtype=torch.int32, device="cuda")
    y = empty(x, ids, out_dtype=torch.float32)
    assert torch.count_nonzero(y) == 0
    with pytest.raises(ValueError, match="range"):
        empty.check()
    assert torch.count_nonzero(empty(x, ids, id_range=(0, 0), out_dtype=torch.float32)) == 0
    empty.check()


def test_activation_output_at_three_tokens():
    h, n, batch = 1024, 900, 3
    gate, up, down = _layer(h, n, torch.bfloat16, seed=21)
    ids = torch.randperm(n, generator=torch.Generator().manual_seed(22))[:300]
    x = torch.randn(batch, h, generator=torch.Generator().manual_seed(23)).bfloat16()
    activation, y = cuda_indexed_parts(x.cuda(), ids.cuda(), gate.cuda(), up.cuda(), down.cuda())
    xs = x.double()
    gv = xs @ gate.double()[ids].T
    uv = xs @ up.double()[ids].T
    a_ref = (gv / (1.0 + torch.exp(-gv)) * uv).numpy()
    assert activation.shape == (batch, ids.numel())
    assert offn.rel_l2(activation.double().cpu().numpy(), a_ref) <= 1e-2
    expected = offn.sparse_ffn_f64(x, ids, gate, up, down)
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-2


def test_oracle_mode_passes_at_six_tokens():
    h, n, tokens = 1024, 2000, 6
    gate, up, down = _layer(h, n, torch.bfloat16, seed=31)
    weights = pack_neuron_major(gate.cuda(), up.cuda(), down.cuda())
    ffn = OracleModeFFN(weights, 0.25, score="activation")
    assert ffn.max_batch == 8
    x = torch.randn(tokens, h, generator=torch.Generator().manual_seed(32)).bfloat16()
    acts = ffn.activations(x.cuda())
    xs = x.double()
    gv = xs @ gate.double().T
    uv = xs @ up.double().T
    a_ref = (gv / (1.0 + torch.exp(-gv)) * uv).numpy()
    assert offn.rel_l2(acts.double().cpu().numpy(), a_ref) <= 1e-5
    ids = ffn.select(acts)
    y = ffn.down(acts, ids, out_dtype=torch.float32)
    a_sel = torch.zeros_like(acts).scatter_(1, ids.long(), acts.gather(1, ids.long())).double().cpu()
    y_ref = (a_sel @ down.double().T).numpy()
    # The activations enter the down MMAs as a 16-bit high part plus its remainder.
    assert offn.rel_l2(y.double().cpu().numpy(), y_ref) <= 1e-5
    ffn.check()


def test_full_size_union_of_eight_tokens():
    layer = workloads.decode_layer(device="cuda")
    n, h = layer.intermediate, layer.hidden
    engine = IndexedSparseFFN(PackedFFNWeights(layer.packed, h, n))
    k = workloads.retention_k(n, 0.05)
    scores = workloads.selector_scores(8, seed=41).cuda()
    union, mask, count = build_union(select_topk(scores, k), 0, n)
    x = workloads.decode_x(batch=8)
    y = engine(x.cuda(), union, token_mask=mask, n_ids_dev=count)
    y32 = engine(x.cuda(), union, token_mask=mask, n_ids_dev=count, out_dtype=torch.float32)
    engine.check()
    m = int(count.item())
    ids = union[:m].long()
    gate = layer.gate().index_select(0, ids).cpu()
    up = layer.up().index_select(0, ids).cpu()
    down = layer.down().index_select(1, ids).cpu()
    expected = offn.sparse_ffn_f64(x, torch.arange(m), gate, up, down, token_mask=mask[:m].cpu())
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-2
    assert offn.rel_l2(y32.double().cpu().numpy(), expected) <= 1e-4
