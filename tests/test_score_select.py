"""Runtime selector score producer: oracle pinned to the reference, host-side folding, ABI checks (CPU)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import predictor as opred
from oracle.select import topk_ids

GOLDEN = Path(__file__).resolve().parent / "golden" / "predictor_cases.npz"
CASES = ["residual", "residual_ref_test", "residual_l64", "factorized"]


def case(name: str) -> dict:
    data = np.load(GOLDEN)
    w = {k.split("/w/", 1)[1]: data[k] for k in data.files if k.startswith(f"{name}/w/")}
    return {"w": w, **{k: data[f"{name}/{k}"] for k in ("mean", "std", "x", "scores", "folded_scores", "k", "ids",
                                                         "ln_eps")}}


def oracle_params(w: dict, mean=None, std=None) -> dict:
    enc_w = w["encoder.weight"].astype(np.float64)
    enc_b = w.get("encoder.bias")
    if std is not None:
        enc_w, shift = opred.fold_normalisation(enc_w, mean, std)
        enc_b = shift if enc_b is None else enc_b + shift
    return {"enc_w": enc_w, "enc_b": enc_b, "fc1_w": w.get("residual_fc1.weight"), "fc1_b": w.get("residual_fc1.bias"),
            "fc2_w": w.get("residual_fc2.weight"), "fc2_b": w.get("residual_fc2.bias"),
            "ln_w": w.get("layer_norm.weight"), "ln_b": w.get("layer_norm.bias"),
            "out_w": w["neurons.weight"], "out_b": w.get("neurons.bias")}


def kind_of(name: str) -> str:
    return "factorized" if name == "factorized" else "residual"


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_runtime_selector(name):
    c = case(name)
    p = oracle_params(c["w"], c["mean"], c["std"])
    scores = opred.predictor_scores(c["x"], p, kind_of(name), float(c["ln_eps"]))
    ref = c["scores"].astype(np.float64)
    assert np.abs(scores - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())
    assert np.abs(c["folded_scores"] - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())
    k = int(c["k"])
    assert k == opred.retention_count(ref.shape[-1], .5)
    ours = topk_ids(scores, k)
    for b in range(ref.shape[0]):
        order = np.sort(ref[b])[::-1]
        if k < ref.shape[1] and order[k - 1] - order[k] <= 1e-4:
            continue  # the boundary is a near tie at fp32 precision
        assert np.array_equal(ours[b], c["ids"][b]), f"row {b}"


class _Predictor(torch.nn.Module):
    """Same attribute names as the reference's residual predictor (predictor/models.py:17-36)."""

    def __init__(self, h, n, latent, residual=True):
        super().__init__()
        self.encoder = torch.nn.Linear(h, latent, bias=False)
        if residual:
            self.residual_fc1 = torch.nn.Linear(latent, latent)
            self.residual_fc2 = torch.nn.Linear(latent, latent)
            self.layer_norm = torch.nn.LayerNorm(latent)
        self.neurons = torch.nn.Linear(latent, n)


def module_from_case(name: str):
    c = case(name)
    h = c["x"].shape[1]
    latent, n = c["w"]["neurons.weight"].shape[1], c["w"]["neurons.weight"].shape[0]
    m = _Predictor(h, n, latent, residual=name != "factorized")
    m.load_state_dict({k: torch.from_numpy(v) for k, v in c["w"].items()})
    return m, c


@pytest.mark.parametrize("name", CASES)
def test_host_folding_matches_reference(name):
    from qcc_b200.runtime.cuda_selector import predictor_params
    m, c = module_from_case(name)
    p, kind, eps = predictor_params(m, torch.from_numpy(c["mean"]), torch.from_numpy(c["std"]))
    host = {k: (None if v is None else v.double().numpy()) for k, v in p.items()}
    scores = opred.predictor_scores(c["x"], host, "factorized" if kind == 1 else "residual", eps)
    ref = c["scores"].astype(np.float64)
    assert np.abs(scores - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())


def test_abi_rejections_without_a_gpu():
    from qcc_b200 import _lib
    lib = _lib.library()
    assert lib.qcc_selector_workspace_bytes(1, 5120, 32, 17408) > 0
    assert lib.qcc_selector_workspace_bytes(1, 5120, 257, 17408) == 0
    assert lib.qcc_selector_workspace_bytes(0, 5120, 32, 17408) == 0

    def call(**kw):
        a = dict(x=1, ldx=16, batch=1, hidden=16, latent=8, n_out=32, kind=0, dtype=_lib.DTYPE_F32, enc_w=1,
                 enc_b=None, fc1_w=1, fc1_b=None, fc2_w=1, fc2_b=None, ln_w=None, ln_b=None, eps=1e-5, out_w=1,
                 out_b=None, k=4, ids=1, ld_ids=4, scores=None, ld_scores=0, ws=16, ws_bytes=0, stream=None)
        a.update(kw)
        return lib.qcc_selector_scores_topk(*a.values())

    assert call(dtype=7) == _lib.ERR_DTYPE
    assert call(kind=2) == _lib.ERR_INVALID_ARGUMENT
    assert call(k=0) == _lib.ERR_SHAPE
    assert call(k=33) == _lib.ERR_SHAPE
    assert call(latent=300) == _lib.ERR_UNSUPPORTED
    assert call(ldx=8) == _lib.ERR_SHAPE
    assert call(fc1_w=None) == _lib.ERR_INVALID_ARGUMENT
    assert call(ws=8, ws_bytes=1 << 20) == _lib.ERR_ALIGNMENT
    assert call(ws_bytes=64) == _lib.ERR_WORKSPACE
    assert call(batch=0) == _lib.OK
