"""CPU restatement of the runtime selector's score producer (test infrastructure only).

The reference's runtime selector scores every neuron with a small predictor
and keeps the top k (runtime/selector.py:15-24, runtime/cuda_selector.py:30-40):

* ``FoldedRuntimeSelector`` (runtime/selector.py:31-38) folds the input
  normalisation (x - mean) / std into the encoder: W' = W / std, b' = -W' mean.
* ``ResidualFactorizedPredictor`` (predictor/models.py:17-36):
  r = silu(E x + e); u = silu(F1 r + f1); v = F2 u + f2 + r;
  z = LayerNorm(v) (biased variance, eps); scores = W z + w.
* ``FactorizedPredictor`` (predictor/models.py:6-14): scores = W (E x) + w.
* ids = ``retention_count`` largest scores (predictor/candidate_reranker.py:9-12),
  returned here with the fixed tie rule of ``oracle.select.topk_ids``.

Everything is float64 numpy on the caller's weight values.
"""
from __future__ import annotations

import math

import numpy as np

from .select import topk_ids


def retention_count(width: int, retention: float) -> int:
    """predictor/candidate_reranker.py:9-12."""
    if not 0 < retention <= 1:
        raise ValueError("retention must be in (0, 1]")
    return max(1, math.ceil(width * retention))


def fold_normalisation(enc_w: np.ndarray, mean: np.ndarray, std: np.ndarray):
    """runtime/selector.py:33-35: encoder weight / std, bias -(W / std) @ mean (std clamped at 1e-6)."""
    std = np.maximum(np.asarray(std, dtype=np.float64), 1e-6)
    w = np.asarray(enc_w, dtype=np.float64) / std[None, :]
    return w, -(w @ np.asarray(mean, dtype=np.float64))


def _silu(v: np.ndarray) -> np.ndarray:
    return v / (1.0 + np.exp(-v))


def predictor_scores(x, p: dict, kind: str = "residual", eps: float = 1e-5) -> np.ndarray:
    """[B, H] -> [B, N] scores (float64).  p holds enc_w, enc_b, fc1_w, fc1_b,
    fc2_w, fc2_b, ln_w, ln_b, out_w, out_b (missing biases count as zero)."""
    f = {k: (None if v is None else np.asarray(v, dtype=np.float64)) for k, v in p.items()}
    x = np.atleast_2d(np.asarray(x, dtype=np.float64))
    pre = x @ f["enc_w"].T
    if f.get("enc_b") is not None:
        pre = pre + f["enc_b"]
    if kind == "factorized":
        z = pre
    elif kind == "residual":
        r = _silu(pre)
        u = _silu(r @ f["fc1_w"].T + (f["fc1_b"] if f.get("fc1_b") is not None else 0.0))
        v = u @ f["fc2_w"].T + (f["fc2_b"] if f.get("fc2_b") is not None else 0.0) + r
        mean = v.mean(axis=-1, keepdims=True)
        var = ((v - mean) ** 2).mean(axis=-1, keepdims=True)
        z = (v - mean) / np.sqrt(var + eps)
        if f.get("ln_w") is not None:
            z = z * f["ln_w"]
        if f.get("ln_b") is not None:
            z = z + f["ln_b"]
    else:
        raise ValueError(f"unknown predictor kind {kind!r}")
    scores = z @ f["out_w"].T
    if f.get("out_b") is not None:
        scores = scores + f["out_b"]
    return scores


def select(x, p: dict, k: int, kind: str = "residual", eps: float = 1e-5) -> np.ndarray:
    """Ascending int32 ids [B, k] of the k largest float64 scores, ties to the lower index."""
    return topk_ids(predictor_scores(x, p, kind, eps), k)


def torch_runtime_selector(x, p: dict, k: int, kind: str = "residual", eps: float = 1e-5):
    """The reference's runtime selector as torch ops on the host (runtime/selector.py:22-24 with the
    predictor forward of predictor/models.py:32-36): scores, then torch.topk(sorted=False).

    Used to time the reference's CPU path; p holds torch tensors (float32)."""
    import torch
    import torch.nn.functional as F

    pre = F.linear(x, p["enc_w"], p.get("enc_b"))
    if kind == "factorized":
        z = pre
    else:
        r = F.silu(pre)
        u = F.silu(F.linear(r, p["fc1_w"], p.get("fc1_b")))
        z = F.layer_norm(r + F.linear(u, p["fc2_w"], p.get("fc2_b")), (r.shape[-1],), p.get("ln_w"), p.get("ln_b"),
                         eps)
    scores = F.linear(z, p["out_w"], p.get("out_b"))
    return torch.topk(scores, k, dim=-1, sorted=False).indices
