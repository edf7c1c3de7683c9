"""Fused indexed FFN on the GPU against the reference's golden outputs and the oracle."""
from __future__ import annotations

import pytest
import torch

from conftest import FFN_CASES, TOL
from oracle import ffn as offn
import qcc_b200.workloads as workloads
from qcc_b200.runtime import IndexedSparseFFN, TorchDynamicSparseFFN, cuda_indexed_ffn, cuda_indexed_parts
from qcc_b200.runtime.packing import pack_neuron_major

pytestmark = pytest.mark.gpu


def _cuda(case, *keys):
    return [case[k].cuda() for k in keys]


@pytest.mark.parametrize("name", FFN_CASES)
@pytest.mark.parametrize("ids_dtype", [torch.int64, torch.int32])
def test_fused_matches_reference_golden(golden_ffn, name, ids_dtype):
    case = golden_ffn[name]
    gate, up, down, x = _cuda(case, "gate", "up", "down", "x")
    ids = case["ids"].to(ids_dtype).cuda()
    y = cuda_indexed_ffn(x, ids, gate, up, down)
    assert y.dtype == x.dtype and y.shape == case["y"].shape
    assert offn.rel_l2(y.double().cpu().numpy(), case["y"].double().numpy()) <= TOL[case["dtype"]]


@pytest.mark.parametrize("name", FFN_CASES)
def test_parts_and_transposed_down(golden_ffn, name):
    case = golden_ffn[name]
    gate, up, down, x = _cuda(case, "gate", "up", "down", "x")
    ids = case["ids"].cuda()
    activation, y = cuda_indexed_parts(x, ids, gate, up, down)
    expected_a = case["activation"] if x.shape[0] > 1 else case["activation"].squeeze(0)
    assert offn.rel_l2(activation.double().cpu().numpy(), expected_a.double().numpy()) <= TOL[case["dtype"]]
    y_t = cuda_indexed_ffn(x, ids, gate, up, down.t().contiguous(), transposed_down=True)
    assert offn.rel_l2(y_t.double().cpu().numpy(), case["y"].double().numpy()) <= TOL[case["dtype"]]


def test_module_drop_in_and_current_stream(golden_ffn):
    # tests/test_phase5b.py:46-50: launches go to the current stream.
    case = golden_ffn["f16_b3"]
    gate, up, down, x = _cuda(case, "gate", "up", "down", "x")
    ids = case["ids"].cuda()
    module = TorchDynamicSparseFFN(gate, up, down)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        y = module(x, ids)
    stream.synchronize()
    assert offn.rel_l2(y.double().cpu().numpy(), case["y"].double().numpy()) <= TOL["float16"]


def test_empty_and_duplicate_ids(golden_ffn):
    case = golden_ffn["small_bf16"]
    gate, up, down, x = _cuda(case, "gate", "up", "down", "x")
    engine = IndexedSparseFFN(pack_neuron_major(gate, up, down))
    y0 = engine(x, torch.empty(0, dtype=torch.int32, device="cuda"))
    assert torch.count_nonzero(y0) == 0
    dup = torch.tensor([3, 3, 7], device="cuda")
    y = engine(x, dup)
    expected = offn.sparse_ffn_f64(case["x"], dup.cpu(), case["gate"], case["up"], case["down"])
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-2


def test_out_of_range_id_is_reported_not_read(golden_ffn):
    case = golden_ffn["small_f32"]
    gate, up, down, x = _cuda(case, "gate", "up", "down", "x")
    engine = IndexedSparseFFN(pack_neuron_major(gate, up, down))
    bad = torch.tensor([1, 5, 96, -3, 10], device="cuda")
    y = engine(x, bad)
    with pytest.raises(ValueError, match="range"):
        engine.check()
    good = torch.tensor([1, 5, 10], device="cuda")
    expected = offn.sparse_ffn_f64(case["x"], good.cpu(), case["gate"], case["up"], case["down"])
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-5
    engine.check()  # status was cleared


def test_batch_chunks_and_token_mask():
    torch.manual_seed(3)
    h, n, b = 256, 300, 7
    gate, up = (torch.randn(n, h) * 0.05).bfloat16(), (torch.randn(n, h) * 0.05).bfloat16()
    down = (torch.randn(h, n) * 0.05).bfloat16()
    x = torch.randn(b, h).bfloat16()
    ids = torch.randperm(n)[:90].sort().values.int()
    mask = torch.randint(0, 128, (90,), dtype=torch.uint8)
    engine = IndexedSparseFFN(pack_neuron_major(gate.cuda(), up.cuda(), down.cuda()))
    y = engine(x.cuda(), ids.cuda(), token_mask=mask.cuda())
    expected = offn.sparse_ffn_f64(x, ids, gate, up, down, token_mask=mask)
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-2
    y32 = engine(x.cuda(), ids.cuda(), token_mask=mask.cuda(), out_dtype=torch.float32)
    assert y32.dtype == torch.float32 and offn.rel_l2(y32.double().cpu().numpy(), expected) <= 1e-4


def test_device_count_limits_ids():
    torch.manual_seed(4)
    h, n = 128, 64
    gate, up, down = (torch.randn(n, h) * .1).float(), (torch.randn(n, h) * .1).float(), (torch.randn(h, n) * .1).float()
    x = torch.randn(1, h)
    ids = torch.arange(0, 40, dtype=torch.int32)
    engine = IndexedSparseFFN(pack_neuron_major(gate.cuda(), up.cuda(), down.cuda()))
    count = torch.tensor([17], dtype=torch.int32, device="cuda")
    y = engine(x.cuda(), ids.cuda(), n_ids_dev=count)
    expected = offn.sparse_ffn_f64(x, ids[:17], gate, up, down)
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-5


@pytest.mark.parametrize("hidden,dtype,batch", [(8192, torch.bfloat16, 2), (5120, torch.float32, 1),
                                                (3000, torch.float16, 3)])
def test_other_hidden_sizes_against_oracle(hidden, dtype, batch):
    torch.manual_seed(5)
    n, k = 700, 175
    gate = (torch.randn(n, hidden) * .02).to(dtype)
    up = (torch.randn(n, hidden) * .02).to(dtype)
    down = (torch.randn(hidden, n) * .02).to(dtype)
    x = torch.randn(batch, hidden).to(dtype)
    ids = torch.randperm(n)[:k]
    y = cuda_indexed_ffn(x.cuda(), ids.cuda(), gate.cuda(), up.cuda(), down.cuda())
    expected = offn.sparse_ffn_f64(x, ids, gate, up, down)
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= (1e-5 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("retention", [0.5, 0.25, 0.1, 0.05])
def test_full_size_decode_against_oracle(retention):
    layer = workloads.decode_layer(device="cuda")
    k = workloads.retention_k(layer.intermediate, retention)
    ids = workloads.decode_ids(layer.intermediate, k)
    x = workloads.decode_x()
    engine = IndexedSparseFFN(pack_neuron_major(layer.gate(), layer.up(), layer.down()))
    y = engine(x.cuda(), ids.cuda())
    # Packed-in-place decode agrees with packing from the three views.
    from qcc_b200.runtime.packing import PackedFFNWeights
    direct = IndexedSparseFFN(PackedFFNWeights(layer.packed, layer.hidden, layer.intermediate))
    y2 = direct(x.cuda(), ids.cuda())
    sel = ids.long().cuda()
    gate = layer.gate().index_select(0, sel).cpu()
    up = layer.up().index_select(0, sel).cpu()
    down_t = layer.packed[:, 2 * layer.hidden:].index_select(0, sel).cpu()
    local = torch.arange(k)
    expected = offn.sparse_ffn_f64(x, local, gate, up, down_t.t())
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= 1e-2
    assert offn.rel_l2(y2.double().cpu().numpy(), expected) <= 1e-2
    # The reference formulation (bf16 rounding between GEMVs) on the same values.
    ref = offn.dynamic_sparse_ffn(x, local, gate, up, down_t.t())
    assert offn.rel_l2(y.double().cpu().numpy(), ref.double().numpy()) <= 1e-2


def test_repeat_calls_reuse_zeroed_workspace(golden_ffn):
    case = golden_ffn["small_f32"]
    gate, up, down, x = _cuda(case, "gate", "up", "down", "x")
    ids = case["ids"].cuda()
    first = cuda_indexed_ffn(x, ids, gate, up, down)
    for _ in range(5):
        again = cuda_indexed_ffn(x, ids, gate, up, down)
    assert offn.rel_l2(again.double().cpu().numpy(), first.double().cpu().numpy()) <= 1e-6


def test_cpu_tensors_fail_loudly(golden_ffn):
    case = golden_ffn["small_f32"]
    with pytest.raises(RuntimeError, match="CUDA"):
        cuda_indexed_ffn(case["x"], case["ids"], case["gate"], case["up"], case["down"])
