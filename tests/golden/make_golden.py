"""Generate the golden fixtures in this directory by running the REFERENCE itself.

Run where robjlyons/qwen-contextual-compression is checked out, naming the
checkout in QCC_REFERENCE (required; there is no default location):

    QCC_REFERENCE=<path to the reference checkout> python tests/golden/make_golden.py

Every expected output below is produced by the reference's own functions
(runtime.ffn, oracle.importance, oracle.sparse_ffn, end_to_end.oracle_sparse_mlp,
runtime.temporal, runtime.selector with predictor.models); inputs are small
seeded tensors.  ``python tests/golden/make_golden.py predictor_cases``
regenerates one fixture only.  The GPU box never runs
this script: it only reads the committed .npz / .json files.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if not os.environ.get("QCC_REFERENCE"):
    raise SystemExit("set QCC_REFERENCE to the reference checkout (robjlyons/qwen-contextual-compression)")
REFERENCE = Path(os.environ["QCC_REFERENCE"])
sys.path.insert(0, str(REFERENCE))
sys.path.append(str(HERE.parents[1]))  # after the reference: its `oracle` package shadows this repo's

from runtime.ffn import DenseFFN, TorchDynamicSparseFFN, masked_dense_reference  # noqa: E402  (reference)
from oracle.importance import block_topk_indices, importance_scores, topk_indices  # noqa: E402  (reference)
from oracle.sparse_ffn import reconstruct  # noqa: E402  (reference)
from end_to_end.oracle_sparse_mlp import OracleSparseMLP  # noqa: E402  (reference)
from runtime.temporal import neuron_payload, simulate_lru_cache  # noqa: E402  (reference)
from runtime.selector import FoldedRuntimeSelector, RuntimeSelector  # noqa: E402  (reference)
from predictor.models import FactorizedPredictor, ResidualFactorizedPredictor  # noqa: E402  (reference)
from predictor.candidate_reranker import retention_count  # noqa: E402  (reference)

import qcc_b200.workloads as workloads  # noqa: E402  (seeded input generators of this repo)


def _raw(t: torch.Tensor) -> np.ndarray:
    """Exact storage of a tensor: bf16 / fp16 as uint16 bits, others as is."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.numpy().view(np.uint16)
    return t.numpy()


def ffn_cases() -> dict:
    out = {}

    def add(name, gate, up, down, x, ids, note):
        ffn = TorchDynamicSparseFFN(gate, up, down)
        y = ffn(x, ids)
        activation = ffn.components(x, ids)[2]
        masked = masked_dense_reference(x, ids, gate, up, down)
        dense_a = DenseFFN(gate, up, down).components(x)[2]
        out[f"{name}/gate"] = _raw(gate)
        out[f"{name}/up"] = _raw(up)
        out[f"{name}/down"] = _raw(down)
        out[f"{name}/x"] = _raw(x)
        out[f"{name}/ids"] = ids.numpy().astype(np.int64)
        out[f"{name}/y"] = _raw(y)
        out[f"{name}/activation"] = _raw(activation)
        out[f"{name}/masked_dense"] = _raw(masked)
        out[f"{name}/dense_activation"] = _raw(dense_a)
        out[f"{name}/dtype"] = np.array(str(gate.dtype).replace("torch.", ""))
        out[f"{name}/note"] = np.array(note)

    # The reference's own unit-test tensors (tests/test_runtime_ffn.py:11-12, 15).
    g = torch.Generator().manual_seed(4)
    gate, up, down, x = (torch.randn(12, 5, generator=g), torch.randn(12, 5, generator=g),
                         torch.randn(5, 12, generator=g), torch.randn(1, 5, generator=g))
    add("reftest_f32", gate, up, down, x, torch.tensor([1, 3, 4, 8, 9, 11]), "tests/test_runtime_ffn.py tensors")

    # The fp16 CUDA test shape (tests/test_phase5b.py:43): seeded here on CPU.
    g = torch.Generator().manual_seed(8)
    x = torch.randn(1, 32, generator=g).half()
    gate = torch.randn(16, 32, generator=g).half()
    up = torch.randn(16, 32, generator=g).half()
    down = torch.randn(32, 16, generator=g).half()
    add("phase5b_f16", gate, up, down, x, torch.tensor([1, 3, 7, 9, 12, 15]), "tests/test_phase5b.py shape, fp16")

    for name, (h, n, k, b, dtype, seed) in {
        "small_f32": (64, 96, 24, 3, torch.float32, 11),
        "small_bf16": (64, 96, 24, 1, torch.bfloat16, 12),
        "pad_bf16": (40, 50, 13, 2, torch.bfloat16, 13),
        "wide_bf16": (1024, 48, 20, 4, torch.bfloat16, 14),
        "f16_b3": (128, 200, 50, 3, torch.float16, 15),
    }.items():
        g = torch.Generator().manual_seed(seed)
        gate = (torch.randn(n, h, generator=g) * 0.1).to(dtype)
        up = (torch.randn(n, h, generator=g) * 0.1).to(dtype)
        down = (torch.randn(h, n, generator=g) * 0.1).to(dtype)
        x = torch.randn(b, h, generator=g).to(dtype)
        ids = torch.randperm(n, generator=g)[:k]  # unsorted, like topk(sorted=False)
        add(name, gate, up, down, x, ids, f"seeded H={h} N={n} K={k} B={b}")
    return out


def select_cases() -> dict:
    out = {}
    # Known answer of tests/test_importance.py:4.
    a = torch.tensor([[1., -4., 2.]])
    w = torch.tensor([[3., 2., 4.], [0., 0., 0.]])
    out["known/scores"] = importance_scores(a, w, "activation").numpy()
    out["known/topk2"] = topk_indices(importance_scores(a, w, "activation"), 2).numpy()

    def tie_rule(scores: torch.Tensor, k: int) -> np.ndarray:
        # The fixed rule the build uses: stable descending sort, first k, ascending.
        order = torch.sort(scores, dim=-1, descending=True, stable=True).indices[:, :k]
        return order.sort(dim=-1).values.numpy().astype(np.int32)

    # Ties, signed zeros, NaN and infinities.
    special = torch.tensor([[0.5, -0.0, 0.0, 0.5, float("nan"), -1.0, 0.5, float("inf"), 0.0, -float("inf"),
                             0.25, 0.5, -0.0, float("nan"), 1e-30, -1e-30]])
    out["special/scores"] = special.numpy()
    for k in (1, 2, 3, 4, 6, 8, 12, 16):
        out[f"special/k{k}"] = tie_rule(special, k)
    # Heavy ties: small integer-valued scores.
    g = torch.Generator().manual_seed(21)
    ties = torch.randint(-3, 4, (3, 257), generator=g).float()
    out["ties/scores"] = ties.numpy()
    for k in (1, 50, 128, 200, 257):
        out[f"ties/k{k}"] = tie_rule(ties, k)
    # Selector workload rows (Laplace + Zipf-boosted hot set) at full N, K/N = 0.2.
    scores = workloads.selector_scores(2)
    k = workloads.retention_k(scores.shape[-1], 0.2)
    expected = tie_rule(scores, k)
    reference = torch.topk(scores, k, dim=-1, sorted=False).indices.sort(dim=-1).values.numpy()
    assert (reference == expected).all(), "no ties at the boundary: reference topk set must equal the tie rule"
    out["workload/scores"] = scores.numpy()
    out["workload/ids"] = expected
    out["workload/k"] = np.array(k)
    # Reference block top-K (oracle/importance.py:26-35) on a tie-free input.
    block_scores = torch.tensor([[1., 1., 9., 9., 2., 2., 0., 0.]])
    out["block/scores"] = block_scores.numpy()
    out["block/k3_b2"] = block_topk_indices(block_scores, 3, 2).numpy()
    g = torch.Generator().manual_seed(22)
    rnd = torch.rand(2, 130, generator=g)
    out["block/rand_scores"] = rnd.numpy()
    out["block/rand_k40_b16"] = block_topk_indices(rnd, 40, 16).numpy()
    return out


class TinyFFN(torch.nn.Module):
    """Same structure as the reference test fixture (tests/conftest.py:5-9)."""

    def __init__(self, h, n):
        super().__init__()
        self.gate_proj = torch.nn.Linear(h, n, bias=False)
        self.up_proj = torch.nn.Linear(h, n, bias=False)
        self.down_proj = torch.nn.Linear(n, h, bias=False)
        self.act_fn = torch.nn.SiLU()

    def forward(self, x):
        return self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x))


def oracle_mlp_cases() -> dict:
    out = {}
    torch.manual_seed(31)
    mlp = TinyFFN(16, 48)
    wrapper = OracleSparseMLP(mlp, 0, 0.25, norm_chunk_columns=7)
    g = torch.Generator().manual_seed(32)
    x = torch.randn(3, 16, generator=g)
    wrapper.set_mode(False)
    dense = wrapper(x)
    wrapper.set_mode(True, 0.25)
    with torch.no_grad():
        sparse = wrapper(x)
    out["gate"] = mlp.gate_proj.weight.detach().numpy()
    out["up"] = mlp.up_proj.weight.detach().numpy()
    out["down"] = mlp.down_proj.weight.detach().numpy()
    out["x"] = x.numpy()
    out["dense"] = dense.detach().numpy()
    out["sparse"] = sparse.detach().numpy()
    out["selected"] = wrapper.last_selected_indices.sort(dim=-1).values.numpy()
    out["norms"] = wrapper.down_column_norms.numpy()
    return out


def lru_cases() -> dict:
    metadata = [{"sample": i, "prompt_id": "p", "token_position": i} for i in range(6)]
    masks = torch.tensor([[0, 1, 2], [1, 2, 3], [4, 5, 6], [1, 4, 7], [0, 1, 2], [2, 3, 8]])
    cases = {}
    for capacity in (0.35, 0.5, 0.75, 1.0):
        result = simulate_lru_cache(masks, metadata, capacity, 12)
        cases[str(capacity)] = {"capacity_neurons": result["capacity_neurons"],
                                "events": [{k: e[k] for k in ("hits", "misses", "evicted", "bytes_transferred",
                                                              "cache_size")} for e in result["events"]]}
    return {"masks": masks.tolist(), "neuron_count": 12, "payload": neuron_payload(), "cases": cases}


def c1_case(tokens: int = 4) -> dict:
    """The CPU oracle workload (hidden 1024, N 3072, fp32), first `tokens` tokens."""
    gate, up, down, x = workloads.oracle_layer()
    x = x[:tokens]
    a = torch.nn.functional.silu(torch.nn.functional.linear(x, gate)) * torch.nn.functional.linear(x, up)
    k = 768
    ids = topk_indices(importance_scores(a, down, "activation"), k)
    y = reconstruct(a, down, ids)
    return {"x": x.numpy(), "ids": ids.sort(dim=-1).values.numpy().astype(np.int32), "y": y.numpy(),
            "k": np.array(k), "checksums": np.array([gate.double().sum().item(), up.double().sum().item(),
                                                     down.double().sum().item(), gate[5, 7].item(),
                                                     down[100, 2000].item()])}


def predictor_cases() -> dict:
    """Scores and selections of the reference's runtime selector (runtime/selector.py:15-38)."""
    out = {}
    shapes = {"residual": (ResidualFactorizedPredictor, 48, 300, 32), "residual_ref_test": (ResidualFactorizedPredictor, 7, 20, 32),
              "residual_l64": (ResidualFactorizedPredictor, 96, 400, 64), "factorized": (FactorizedPredictor, 48, 300, 64)}
    for i, (name, (cls, h, n, latent)) in enumerate(shapes.items()):
        torch.manual_seed(40 + i)
        model = cls(h, n, latent).eval()
        with torch.no_grad():  # non-trivial LayerNorm affine and biases
            for prm in model.parameters():
                prm.add_(0.05 * torch.randn_like(prm))
        mean, std = torch.randn(h), torch.rand(h) + .2
        x = torch.randn(4, h)
        base = RuntimeSelector(model, mean, std, .5)
        folded = FoldedRuntimeSelector(model, mean, std, .5, torch.float32)
        with torch.no_grad():
            scores = base.scores(x)
            folded_scores = folded.scores(x)
        k = retention_count(n, .5)
        for key, t in model.state_dict().items():
            out[f"{name}/w/{key}"] = t.numpy()
        out[f"{name}/mean"], out[f"{name}/std"], out[f"{name}/x"] = mean.numpy(), std.numpy(), x.numpy()
        out[f"{name}/scores"], out[f"{name}/folded_scores"] = scores.numpy(), folded_scores.numpy()
        out[f"{name}/k"] = np.array(k)
        out[f"{name}/ids"] = torch.sort(scores, dim=-1, descending=True, stable=True).indices[:, :k].sort(
            dim=-1).values.numpy().astype(np.int32)
        out[f"{name}/ln_eps"] = np.array(getattr(getattr(model, "layer_norm", None), "eps", 1e-5))
    return out


FIXTURES = {"ffn_cases": ffn_cases, "select_cases": select_cases, "oracle_mlp": oracle_mlp_cases,
            "c1_oracle": c1_case, "predictor_cases": predictor_cases}


def main() -> None:
    only = [a for a in sys.argv[1:] if not a.startswith("-")]
    if only:  # regenerate just these fixtures
        for name in only:
            np.savez_compressed(HERE / f"{name}.npz", **FIXTURES[name]())
            print(name, (HERE / f"{name}.npz").stat().st_size)
        return
    np.savez_compressed(HERE / "predictor_cases.npz", **predictor_cases())
    np.savez_compressed(HERE / "ffn_cases.npz", **ffn_cases())
    np.savez_compressed(HERE / "select_cases.npz", **select_cases())
    np.savez_compressed(HERE / "oracle_mlp.npz", **oracle_mlp_cases())
    np.savez_compressed(HERE / "c1_oracle.npz", **c1_case())
    (HERE / "lru_cases.json").write_text(json.dumps(lru_cases(), indent=1))
    (HERE / "PROVENANCE.json").write_text(json.dumps({
        "generator": "tests/golden/make_golden.py", "torch": torch.__version__, "numpy": np.__version__,
        "reference": "robjlyons/qwen-contextual-compression (runtime/ffn.py, oracle/importance.py, "
                     "oracle/sparse_ffn.py, end_to_end/oracle_sparse_mlp.py, runtime/temporal.py, "
                     "runtime/selector.py, predictor/models.py)"}, indent=1))
    for path in sorted(HERE.glob("*.npz")):
        print(path.name, path.stat().st_size)


if __name__ == "__main__":
    main()
