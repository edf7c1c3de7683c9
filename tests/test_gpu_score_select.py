"""Fused score producer + top-K (qcc_selector_scores_topk) against the oracle, on the GPU."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import predictor as opred
from oracle.select import topk_ids
from tests.test_score_select import CASES, case, kind_of, module_from_case, oracle_params

pytestmark = pytest.mark.gpu

SCORE_TOL = 1e-4  # fp32 arithmetic on the same weight values vs float64


def _engine(p: dict, kind: int, k: int, dtype=torch.float32, eps=1e-5):
    from qcc_b200.runtime.cuda_selector import FusedScoreSelector
    t = {name: (None if v is None else torch.as_tensor(np.asarray(v, dtype=np.float32))) for name, v in p.items()}
    return FusedScoreSelector(t, kind=kind, k=k, eps=eps, dtype=dtype, device="cuda")


def _rounded(p: dict, dtype) -> dict:
    """The weight values the engine holds after casting to dtype, as float64."""
    return {n: (None if v is None else torch.as_tensor(np.asarray(v, dtype=np.float32)).to(dtype).double().numpy())
            for n, v in p.items()}


def _check_selection(ids: np.ndarray, gpu_scores: np.ndarray, ref_scores: np.ndarray, k: int):
    # Selection is exact on the kernel's own scores ...
    assert np.array_equal(ids, topk_ids(gpu_scores, k))
    # ... and equals the oracle's wherever the boundary is not a near tie.
    expect = topk_ids(ref_scores, k)
    for b in range(ids.shape[0]):
        order = np.sort(ref_scores[b])[::-1]
        if k < ref_scores.shape[1] and order[k - 1] - order[k] <= 1e-3 * max(1.0, abs(order[k])):
            continue
        assert np.array_equal(ids[b], expect[b]), f"row {b}"


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_reference_cases(name, dtype):
    c = case(name)
    p = oracle_params(c["w"], c["mean"], c["std"])
    kind = 1 if name == "factorized" else 0
    k = int(c["k"])
    eng = _engine(p, kind, k, dtype, float(c["ln_eps"]))
    x = torch.as_tensor(c["x"]).cuda()
    scores, ids = eng.run(x)
    eng.check()
    xr = x.to(dtype).double().cpu().numpy()
    ref = opred.predictor_scores(xr, _rounded(p, dtype), kind_of(name), float(c["ln_eps"]))
    got = scores.double().cpu().numpy()
    assert np.abs(got - ref).max() <= SCORE_TOL * max(1.0, np.abs(ref).max())
    _check_selection(ids.cpu().numpy(), scores.cpu().numpy(), ref, k)
    if dtype == torch.float32:
        # Against the reference's own scores and ids (tests/golden, made by the reference).
        assert np.abs(got - c["scores"]).max() <= SCORE_TOL * max(1.0, np.abs(c["scores"]).max())


@pytest.mark.parametrize("batch", [1, 3, 40])
@pytest.mark.parametrize("k_frac", [0.5, 0.2, 1.0])
def test_cuda_selector_shape(batch, k_frac):
    """The reference CudaSelector's shape: hidden 5120, latent 32, 17408 neurons."""
    g = torch.Generator().manual_seed(7)
    h, latent, n = 5120, 32, 17408
    p = {"enc_w": torch.randn(latent, h, generator=g) * 0.02, "enc_b": torch.randn(latent, generator=g) * 0.1,
         "fc1_w": torch.randn(latent, latent, generator=g) * 0.2, "fc1_b": torch.randn(latent, generator=g) * 0.1,
         "fc2_w": torch.randn(latent, latent, generator=g) * 0.2, "fc2_b": torch.randn(latent, generator=g) * 0.1,
         "ln_w": 1 + 0.1 * torch.randn(latent, generator=g), "ln_b": 0.1 * torch.randn(latent, generator=g),
         "out_w": torch.randn(n, latent, generator=g) * 0.2, "out_b": torch.randn(n, generator=g) * 0.1}
    k = opred.retention_count(n, k_frac)
    eng = _engine({a: b.numpy() for a, b in p.items()}, 0, k, torch.bfloat16)
    x = torch.randn(batch, h, generator=g).cuda()
    scores, ids = eng.run(x)
    eng.check()
    ref = opred.predictor_scores(x.to(torch.bfloat16).double().cpu().numpy(),
                                 _rounded({a: b.numpy() for a, b in p.items()}, torch.bfloat16), "residual")
    got = scores.double().cpu().numpy()
    assert np.abs(got - ref).max() <= SCORE_TOL * max(1.0, np.abs(ref).max())
    _check_selection(ids.cpu().numpy(), scores.cpu().numpy(), ref, k)
    # Calls leave the workspace clean: a second call gives the same ids.
    assert torch.equal(eng.select(x), ids)


def test_exact_ties_take_the_lower_index():
    """A zero head: every score is its bias; integer biases tie exactly."""
    n, h, latent = 5000, 64, 32
    g = torch.Generator().manual_seed(3)
    bias = torch.randint(-3, 4, (n,), generator=g).float()
    p = {"enc_w": torch.randn(latent, h, generator=g).numpy(), "enc_b": None, "out_w": np.zeros((n, latent),
                                                                                                 np.float32),
         "out_b": bias.numpy()}
    x = torch.randn(2, h, generator=g).cuda()
    for k in (1, 700, 2500, 4999, 5000):
        eng = _engine(p, 1, k)
        scores, ids = eng.run(x)
        expect = topk_ids(np.broadcast_to(bias.numpy(), (2, n)), k)
        assert np.array_equal(ids.cpu().numpy(), expect), k
        assert torch.equal(scores.cpu(), bias.expand(2, n))


def test_mirrors_of_the_reference_classes():
    from qcc_b200.runtime.cuda_selector import CudaSelector, RuntimeSelector
    m, c = module_from_case("residual")
    sel = RuntimeSelector(m, torch.from_numpy(c["mean"]), torch.from_numpy(c["std"]), .5)
    x = torch.as_tensor(c["x"]).cuda()
    ids = sel.select(x).cpu().numpy()
    ref = c["scores"].astype(np.float64)
    _check_selection(ids, sel.scores(x).cpu().numpy(), ref, int(c["k"]))

    class Folded:  # the reference CudaSelector reads .predictor of a folded selector
        predictor = m
    cuda = CudaSelector(Folded())
    assert cuda.k == m.neurons.out_features // 2
    raw = opred.predictor_scores(c["x"], oracle_params(c["w"]), "residual")
    got = cuda.scores(x).double().cpu().numpy()
    assert np.abs(got - raw).max() <= SCORE_TOL * max(1.0, np.abs(raw).max())
    with pytest.raises(ValueError, match="batch"):
        cuda.scores(x[0])


@pytest.mark.parametrize("n,latent,dtype", [
    (40000, 32, torch.bfloat16),   # beyond one cluster's shared memory: the grid-wide kernel
    (17408, 64, torch.float32),    # cluster kernel, head rows read from global memory
    (17408, 36, torch.float16),    # latent not a multiple of 8: scalar weight rows
])
def test_both_kernel_paths(n, latent, dtype):
    g = torch.Generator().manual_seed(n + latent)
    h = 1000
    p = {"enc_w": torch.randn(latent, h, generator=g) * 0.05, "enc_b": torch.randn(latent, generator=g) * 0.1,
         "fc1_w": torch.randn(latent, latent, generator=g) * 0.2, "fc1_b": torch.randn(latent, generator=g) * 0.1,
         "fc2_w": torch.randn(latent, latent, generator=g) * 0.2, "fc2_b": None,
         "ln_w": 1 + 0.1 * torch.randn(latent, generator=g), "ln_b": None,
         "out_w": torch.randn(n, latent, generator=g) * 0.2, "out_b": torch.randn(n, generator=g) * 0.1}
    p = {a: (None if b is None else b.numpy()) for a, b in p.items()}
    k = opred.retention_count(n, 0.3)
    eng = _engine(p, 0, k, dtype)
    x = torch.randn(2, h, generator=g).cuda()
    for _ in range(2):  # the second call checks the workspace was left clean
        scores, ids = eng.run(x)
        eng.check()
        ref = opred.predictor_scores(x.to(dtype).double().cpu().numpy(), _rounded(p, dtype), "residual")
        got = scores.double().cpu().numpy()
        assert np.abs(got - ref).max() <= SCORE_TOL * max(1.0, np.abs(ref).max())
        _check_selection(ids.cpu().numpy(), scores.cpu().numpy(), ref, k)
