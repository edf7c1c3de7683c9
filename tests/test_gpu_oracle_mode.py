"""Oracle-mode FFN on the GPU: activations, activation top-K, indexed down, and the C1 workload.

* C1 (the CPU-runnable oracle configuration: hidden 1024, N 3072, fp32, 64
  RMS-normalised tokens, per-token top-K of |silu(g) * u| at K/N = 0.25,
  y = D[:, ids] a[ids]) runs through the product path -- gate/up pass,
  activation top-K, down pass -- and is compared with the reference's own
  outputs (tests/golden/c1_oracle.npz, first tokens: ids bit for bit, y within
  1e-5) and with the oracle for every token.
* Each kernel against the oracle on its own: activations within the dtype's
  tolerance of float64, the selection bit-exact against the tie rule applied
  to the same fp32 scores (bf16 / fp16 / fp32 rows, with and without column
  weights, ties, k = 1 and k = n), the masked row exact, and the down pass
  within tolerance of float64 with per-token token bits.
* The full layer size (hidden 5120, N 17408, bf16, 4 tokens, |a| * ||D||).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import TOL, load_npz
from oracle import ffn as offn
from oracle.select import topk_ids
import qcc_b200.workloads as workloads
from qcc_b200.runtime.oracle_mode import OracleModeFFN, down_column_norms
from qcc_b200.runtime.packing import PackedFFNWeights, pack_neuron_major
from qcc_b200.runtime.selector import activation_topk

pytestmark = pytest.mark.gpu


def _near_tie(scores: np.ndarray, k: int, rel: float = 1e-5) -> bool:
    order = np.sort(scores)[::-1]
    return k < scores.size and order[k - 1] - order[k] <= rel * max(1.0, abs(order[k]))


def test_c1_oracle_workload_through_the_gpu_path():
    data = load_npz("c1_oracle.npz")
    gate, up, down, x = workloads.oracle_layer()
    k = int(data["k"])
    weights = pack_neuron_major(gate.cuda(), up.cuda(), down.cuda())
    ffn = OracleModeFFN(weights, retention=0.25, score="activation")
    assert ffn.k == k
    y, ids = ffn(x.cuda(), out_dtype=torch.float32)
    torch.cuda.synchronize()
    ffn.check()
    ids = ids.cpu().numpy()
    golden_tokens = data["x"].shape[0]
    # The reference's own outputs for the first tokens.
    assert np.array_equal(ids[:golden_tokens], data["ids"])
    np.testing.assert_allclose(y[:golden_tokens].cpu().numpy(), data["y"], rtol=1e-5, atol=1e-6)
    # Every token against the oracle (fp32 torch activations, the tie rule).
    a = torch.nn.functional.silu(x @ gate.T) * (x @ up.T)
    scores = offn.importance_scores(a, down, "activation").numpy()
    want = topk_ids(scores, k)
    # The kernel's fp32 activations and torch's differ in summation order: a
    # token may only choose differently where its K-th and (K+1)-th scores lie
    # within that rounding noise of each other.
    for t in range(x.shape[0]):
        if not np.array_equal(ids[t], want[t]):
            assert _near_tie(scores[t], k, rel=1e-6), f"token {t}"
    y_ref = offn.reconstruct(a, down, torch.from_numpy(ids).long())
    assert offn.rel_l2(y.cpu().numpy(), y_ref.numpy()) <= TOL["float32"]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tokens", [1, 3, 6])
def test_activations_pass_matches_f64(dtype, tokens):
    hidden, n = 768, 1000
    gate, up, down, x = workloads.oracle_layer(hidden, n, tokens, seed=3)
    gate, up, down, x = (t.to(dtype) for t in (gate, up, down, x))
    ffn = OracleModeFFN(pack_neuron_major(gate.cuda(), up.cuda(), down.cuda()), 0.3, score="activation")
    acts = ffn.activations(x.cuda()).cpu().double().numpy()
    xs, g, u = x.double().numpy(), gate.double().numpy(), up.double().numpy()
    gv, uv = xs @ g.T, xs @ u.T
    want = gv / (1 + np.exp(-gv)) * uv
    assert np.abs(acts - want).max() <= 1e-5 * np.abs(want).max()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("weighted", [False, True])
def test_activation_topk_is_the_tie_rule_on_the_same_scores(dtype, weighted):
    g = torch.Generator().manual_seed(11)
    rows, n = 5, 4099
    act = torch.randn(rows, n, generator=g).to(dtype)
    act[1, 100:300] = act[1, 99]           # exact ties across the boundary
    act[2, :] = 0.0
    act[2, 7] = -0.0
    w = (0.5 + torch.rand(n, generator=g)) if weighted else None
    for k in (1, 37, 1000, n):
        ids, masked = activation_topk(act.cuda(), k, None if w is None else w.cuda(), masked=True)
        scores = act.float().abs() * (w if weighted else 1.0)
        want = topk_ids(scores.numpy(), k)
        assert np.array_equal(ids.cpu().numpy(), want), f"k={k}"
        keep = torch.zeros(rows, n, dtype=torch.bool)
        keep.scatter_(1, torch.from_numpy(want).long(), True)
        assert torch.equal(masked.cpu(), torch.where(keep, act, torch.zeros_like(act)))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("tokens", [1, 2, 4])
def test_down_pass_matches_f64_with_token_bits(dtype, tokens):
    hidden, n = 1024, 1536
    gate, up, down, x = workloads.oracle_layer(hidden, n, tokens, seed=5)
    gate, up, down, x = (t.to(dtype) for t in (gate, up, down, x))
    ffn = OracleModeFFN(pack_neuron_major(gate.cuda(), up.cuda(), down.cuda()), 0.2, score="weighted_activation")
    acts = ffn.activations(x.cuda())
    ids = ffn.select(acts)
    y = ffn.down(acts, ids, out_dtype=torch.float32).cpu().double().numpy()
    a = acts.cpu().double().numpy()
    d = down.double().numpy()
    for t in range(tokens):
        sel = ids[t].cpu().long().numpy()
        want = d[:, sel] @ a[t, sel]
        assert offn.rel_l2(y[t], want) <= 1e-5
    # Norm weights: ||D[:, j]|| of the packed down parts against float64 norms (the
    # weights' fp32 rounding is the only error left: sums are accumulated in fp64).
    np.testing.assert_allclose(down_column_norms(ffn.weights).cpu().numpy(),
                               np.linalg.norm(down.double().numpy(), axis=0), rtol=1e-7)


def test_full_layer_size_weighted():
    hidden, n, tokens = workloads.DECODE_HIDDEN, workloads.DECODE_INTERMEDIATE, 4
    layer = workloads.decode_layer(device="cuda", seed=77)
    ffn = OracleModeFFN(PackedFFNWeights(layer.packed, hidden, n), 0.25, score="weighted_activation")
    x = workloads.decode_x(batch=tokens, seed=6).cuda()
    y, ids = ffn(x)
    torch.cuda.synchronize()
    ffn.check()
    gate, up, down = layer.gate().cpu(), layer.up().cpu(), layer.down().cpu()
    xs = x.cpu().double().numpy()
    gv = xs @ gate.double().numpy().T
    uv = xs @ up.double().numpy().T
    a = gv / (1 + np.exp(-gv)) * uv
    norms = np.linalg.norm(down.double().numpy(), axis=0)
    scores = np.abs(a) * norms
    ids = ids.cpu().numpy()
    for t in range(tokens):
        # The kernel's fp32 scores and float64 ones may order a near tie differently;
        # everything clear of the boundary must agree.
        want = set(topk_ids(scores[t:t + 1], ffn.k)[0].tolist())
        got = set(ids[t].tolist())
        order = np.sort(scores[t])[::-1]
        boundary = order[ffn.k - 1]
        clear = {j for j in want if scores[t, j] > boundary * (1 + 1e-4)}
        assert clear <= got
        assert len(want ^ got) <= 8
        y_ref = offn.sparse_ffn_f64(x[t:t + 1].cpu(), torch.from_numpy(ids[t]).long(), gate, up, down)
        assert offn.rel_l2(y[t:t + 1].double().cpu().numpy(), y_ref) <= TOL["bfloat16"]
