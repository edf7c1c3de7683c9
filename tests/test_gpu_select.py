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


def _expand(blocks: np.ndarray, block: int, n: int) -> np.ndarray:
    """Block ids -> neuron ids the way reference oracle/importance.py:32-35 expands them."""
    idx = (blocks.astype(np.int64)[..., None] * block + np.arange(block)).reshape(blocks.shape[0], -1)
    idx = np.where(idx >= n, n, idx)
    return np.sort(idx, axis=-1)[:, :min(blocks.shape[-1] * block, n)]


def test_block_topk_matches_reference_golden():
    from qcc_b200.runtime.selector import block_topk

    data = load_npz("select_cases.npz")
    for scores, k, block, key in ((data["block/scores"], 3, 2, "block/k3_b2"),
                                  (data["block/rand_scores"], 40, 16, "block/rand_k40_b16")):
        blocks = block_topk(torch.from_numpy(scores).cuda(), k, block).cpu().numpy()
        assert np.array_equal(_expand(blocks, block, scores.shape[-1]), data[key])


@pytest.mark.parametrize("n,k,block,rows", [(17408, 5222, 64, 8), (1000, 100, 16, 3), (130, 130, 16, 2),
                                            (4099, 1, 64, 4)])
def test_block_topk_against_oracle(n, k, block, rows):
    from qcc_b200.runtime.selector import block_topk

    gen = torch.Generator().manual_seed(n + k)
    scores = torch.randn(rows, n, generator=gen).abs()
    scores[:, 64:128] = scores[:, 0:64]  # two blocks with the same sum: a tie
    blocks, sums = block_topk(scores.cuda(), k, block, with_sums=True)
    blocks, sums = blocks.cpu().numpy(), sums.cpu().numpy()
    nb = (n + block - 1) // block
    padded = np.zeros((rows, nb * block))
    padded[:, :n] = scores.double().numpy()
    want_sums = padded.reshape(rows, nb, block).sum(-1)
    np.testing.assert_allclose(sums, want_sums, rtol=1e-6)
    kb = max(1, min(nb, (k + block - 1) // block))
    # Selection is exact on the kernel's sums; and equals the oracle's expansion.
    assert np.array_equal(blocks, osel.topk_ids(sums, kb))
    oracle = osel.block_topk_indices(scores.numpy(), k, block)
    for r in range(rows):  # the oracle sums in float32; only a near tie may order differently
        order = np.sort(want_sums[r])[::-1]
        if kb < nb and order[kb - 1] - order[kb] <= 1e-5 * order[kb]:
            continue
        assert np.array_equal(_expand(blocks[r:r + 1], block, n)[0], oracle[r])


def test_scores_to_prefill_tiles_end_to_end():
    """Token scores -> block top-K -> per-tile unions -> block-sparse prefill, against host-built lists."""
    from qcc_b200.runtime.packing import PackedFFNWeights
    from qcc_b200.runtime.prefill import BlockSparsePrefill, tile_block_lists
    from qcc_b200.runtime.selector import block_topk, tile_block_union

    hidden, n, tokens, block = 1024, 4096, 300, 64
    layer = workloads.decode_layer(hidden=hidden, intermediate=n, device="cuda", seed=8)
    gen = torch.Generator().manual_seed(4)
    scores = torch.randn(tokens, n, generator=gen).abs()
    blocks = block_topk(scores.cuda(), 640, block)  # 10 of 64 blocks per token
    flat, offsets = tile_block_union(blocks, n // block, tile_rows=128)
    host = blocks.cpu().numpy()
    tiles = [np.unique(host[t:t + 128]) for t in range(0, tokens, 128)]
    off = offsets.cpu().numpy()
    assert off[0] == 0 and len(off) == len(tiles) + 1
    for t, want in enumerate(tiles):
        assert np.array_equal(flat[off[t]:off[t + 1]].cpu().numpy(), want)
    engine = BlockSparsePrefill(PackedFFNWeights(layer.packed, hidden, n))
    x = workloads.prefill_x(tokens=tokens, hidden=hidden).cuda()
    y_dev = engine(x, (flat, offsets))
    y_host = engine(x, tile_block_lists([torch.from_numpy(t) for t in tiles], x.device))
    torch.cuda.synchronize()
    engine.check()
    assert torch.equal(y_dev, y_host)
