"""Pin the CPU oracle to golden vectors produced by the reference itself."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import FFN_CASES, TOL, load_json, load_npz
from oracle import ffn as offn
from oracle import lru as olru
from oracle import select as osel


@pytest.mark.parametrize("name", FFN_CASES)
def test_oracle_ffn_reproduces_reference_bits(golden_ffn, name):
    case = golden_ffn[name]
    y = offn.dynamic_sparse_ffn(case["x"], case["ids"], case["gate"], case["up"], case["down"])
    # Same ATen sequence on the same CPU: identical bits.
    assert torch.equal(y, case["y"])
    a = offn.dynamic_sparse_activation(case["x"], case["ids"], case["gate"], case["up"])
    assert torch.equal(a, case["activation"])
    masked = offn.masked_dense(case["x"], case["ids"], case["gate"], case["up"], case["down"])
    assert torch.equal(masked, case["masked_dense"])


@pytest.mark.parametrize("name", FFN_CASES)
def test_f64_oracle_within_tolerance_of_reference(golden_ffn, name):
    case = golden_ffn[name]
    y64 = offn.sparse_ffn_f64(case["x"], case["ids"], case["gate"], case["up"], case["down"])
    assert offn.rel_l2(case["y"].double().numpy(), y64) <= TOL[case["dtype"]]


def test_dense_activation_indexed_equals_sparse_activation(golden_ffn):
    # tests/test_runtime_ffn.py:15: dense components at ids equal the sparse ones.
    case = golden_ffn["reftest_f32"]
    torch.testing.assert_close(case["dense_activation"][:, case["ids"]], case["activation"])


def test_pack_records_layout(golden_ffn):
    case = golden_ffn["pad_bf16"]
    gate, up, down = (case[k].float().numpy() for k in ("gate", "up", "down"))
    packed = offn.pack_records(gate, up, down)
    n, h = gate.shape
    hp = (h + 7) // 8 * 8
    assert packed.shape == (n, 3 * hp)
    assert np.array_equal(packed[7, :h], gate[7]) and np.array_equal(packed[7, hp:hp + h], up[7])
    assert np.array_equal(packed[7, 2 * hp:2 * hp + h], down[:, 7])
    assert not packed[:, h:hp].any() and not packed[:, 3 * hp - (hp - h):].any()


def test_selection_known_answer():
    data = load_npz("select_cases.npz")
    assert osel.topk_ids(data["known/scores"], 2).tolist() == [[1, 2]]
    assert np.array_equal(np.sort(data["known/topk2"], -1), [[1, 2]])


@pytest.mark.parametrize("group,ks", [("special", (1, 2, 3, 4, 6, 8, 12, 16)), ("ties", (1, 50, 128, 200, 257))])
def test_selection_tie_rule_matches_golden(group, ks):
    data = load_npz("select_cases.npz")
    for k in ks:
        assert np.array_equal(osel.topk_ids(data[f"{group}/scores"], k), data[f"{group}/k{k}"]), k


def test_selection_workload_rows_match_reference_topk_set():
    data = load_npz("select_cases.npz")
    k = int(data["workload/k"])
    assert np.array_equal(osel.topk_ids(data["workload/scores"], k), data["workload/ids"])


def test_block_topk_matches_reference():
    data = load_npz("select_cases.npz")
    assert np.array_equal(osel.block_topk_indices(data["block/scores"], 3, 2), data["block/k3_b2"])
    assert np.array_equal(osel.block_topk_indices(data["block/rand_scores"], 40, 16), data["block/rand_k40_b16"])


def test_signed_zero_and_nan_keys():
    keys = osel.score_keys(np.array([-0.0, 0.0, np.nan, -np.nan, np.inf, -np.inf, 1.0, -1.0], dtype=np.float32))
    assert keys[0] == keys[1]
    assert keys[2] == keys[3] == 0xFFFFFFFF
    assert keys[4] > keys[6] > keys[0] > keys[7] > keys[5]


def test_union_with_mask():
    rows = np.array([[1, 4, 9], [4, 5, 9], [0, 9, 11]])
    ids, mask = osel.union_with_mask(rows, 3, 10)
    assert ids.tolist() == [1, 2, 6]          # 4, 5, 9 rebased by 3
    assert mask.tolist() == [0b011, 0b010, 0b111]


def test_lru_accounting_matches_reference():
    data = load_json("lru_cases.json")
    assert olru.neuron_payload() == data["payload"] == 30720
    for case in data["cases"].values():
        events = olru.lru_events(data["masks"], case["capacity_neurons"])
        assert events == case["events"]


def test_c1_oracle_workload():
    import qcc_b200.workloads as workloads
    data = load_npz("c1_oracle.npz")
    gate, up, down, x = workloads.oracle_layer()
    sums = np.array([gate.double().sum().item(), up.double().sum().item(), down.double().sum().item(),
                     gate[5, 7].item(), down[100, 2000].item()])
    np.testing.assert_allclose(sums, data["checksums"], rtol=0, atol=0)
    tokens = data["x"].shape[0]
    assert np.array_equal(x[:tokens].numpy(), data["x"])
    a = torch.nn.functional.silu(x[:tokens] @ gate.T) * (x[:tokens] @ up.T)
    ids = osel.topk_ids(offn.importance_scores(a, down, "activation").numpy(), int(data["k"]))
    assert np.array_equal(ids, data["ids"])
    y = offn.reconstruct(a, down, torch.from_numpy(ids).long())
    np.testing.assert_allclose(y.numpy(), data["y"], rtol=1e-5, atol=1e-6)
