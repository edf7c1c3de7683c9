"""GPU selector and union kernels, bit-exact against the oracle and the golden ids."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_npz
from oracle import select as osel
from qcc_b200.runtime.selector import TopKSelector, build_union, select_topk
import qcc_b200.workloads as workloads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("group,ks", [("special", (1, 2, 3, 4, 6, 8, 12, 16)), ("ties", (1, 50, 128, 200, 257))])
def test_tie_rule_bit_exact(group, ks):
    data = load_npz("select_cases.npz")
    scores = torch.from_numpy(data[f"{group}/scores"]).cuda()
    for k in ks:
        ids = select_topk(scores, k).cpu().numpy()
        assert np.array_equal(ids, data[f"{group}/k{k}"]), k


def test_workload_rows_match_reference():
    data = load_npz("select_cases.npz")
    k = int(data["workload/k"])
    ids = select_topk(torch.from_numpy(data["workload/scores"]).cuda(), k).cpu().numpy()
    assert np.array_equal(ids, data["workload/ids"])


@pytest.mark.parametrize("n,k,batch", [(17408, 4352, 1), (17408, 3482, 8), (1000, 1, 3), (1000, 1000, 2),
                                       (33, 7, 5), (50000, 12345, 2)])
def test_random_rows_against_oracle(n, k, batch):
    gen = torch.Generator().manual_seed(n + k)
    scores = torch.randn(batch, n, generator=gen)
    scores[:, ::7] = scores[:, 3:4]  # plant ties
    ids = select_topk(scores.cuda(), k).cpu().numpy()
    assert np.array_equal(ids, osel.topk_ids(scores.numpy(), k))


def test_selector_workload_and_k_zero():
    scores = workloads.selector_scores(4)
    selector = TopKSelector(scores.shape[-1], 0.2)
    ids = selector.select(scores.cuda()).cpu().numpy()
    assert ids.shape == (4, 3482)
    assert np.array_equal(ids, osel.topk_ids(scores.numpy(), 3482))
    assert select_topk(scores.cuda(), 0).shape == (4, 0)


@pytest.mark.parametrize("begin,end", [(0, 17408), (4352, 8704), (17000, 17408)])
def test_union_against_oracle(begin, end):
    scores = workloads.selector_scores(5)
    rows = osel.topk_ids(scores.numpy(), 3482)
    union, mask, count = build_union(torch.from_numpy(rows).cuda(), begin, end)
    expected_ids, expected_mask = osel.union_with_mask(rows, begin, end)
    c = int(count.item())
    assert c == len(expected_ids)
    assert np.array_equal(union[:c].cpu().numpy(), expected_ids)
    assert np.array_equal(mask[:c].cpu().numpy(), expected_mask)
