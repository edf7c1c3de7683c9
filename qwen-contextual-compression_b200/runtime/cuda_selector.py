"""Fused score producer + top-K: the reference's runtime selector in one launch.

Mirrors reference runtime/cuda_selector.py:45-51 (``CudaSelector``: fused
latent + head kernels, then ``torch.topk(scores, k, sorted=False)`` with
k = out_features // 2) and runtime/selector.py:15-38 (``RuntimeSelector`` /
``FoldedRuntimeSelector``: normalise x, score with the predictor, keep
``retention_count`` neurons).  Here one ``qcc_selector_scores_topk`` launch
computes the predictor (encoder with the normalisation folded in, residual
MLP, LayerNorm, neuron head) and the deterministic top-K: ids come back as
ascending int32, ties to the lower index; scores are fp32.

Predictors are read through their attributes, as the reference's kernels do:
``encoder``, ``residual_fc1``, ``residual_fc2``, ``layer_norm``, ``neurons``
(predictor/models.py:17-36) or ``encoder`` + ``neurons`` only
(predictor/models.py:6-14).  There is no CPU fallback.
"""
from __future__ import annotations

import math
import threading

import torch

from .. import _lib

KIND_RESIDUAL, KIND_FACTORIZED = 0, 1
_MAX_LATENT = 256


def retention_count(width: int, retention: float) -> int:
    """predictor/candidate_reranker.py:9-12."""
    if not 0 < retention <= 1:
        raise ValueError("retention must be in (0, 1]")
    return max(1, math.ceil(width * retention))


def _param(module, name):
    t = getattr(module, name, None)
    return None if t is None else t.detach()


def predictor_params(predictor, mean=None, std=None) -> tuple[dict, int, float]:
    """(weights, kind, LayerNorm eps) of a residual or factorized predictor.

    mean / std (the checkpoint normalisation of runtime/selector.py:15-20) are
    folded into the encoder as runtime/selector.py:33-35 does: W / std, bias
    b - (W / std) mean (std clamped at 1e-6).
    """
    enc_w = predictor.encoder.weight.detach().float()
    enc_b = _param(predictor.encoder, "bias")
    enc_b = None if enc_b is None else enc_b.float()
    if std is not None:
        enc_w = enc_w / std.detach().float().clamp_min(1e-6).to(enc_w.device)[None, :]
    if mean is not None:
        shift = -(enc_w @ mean.detach().float().to(enc_w.device))
        enc_b = shift if enc_b is None else enc_b + shift
    p = {"enc_w": enc_w, "enc_b": enc_b, "out_w": predictor.neurons.weight.detach(),
         "out_b": _param(predictor.neurons, "bias")}
    if hasattr(predictor, "residual_fc1"):
        p.update(fc1_w=predictor.residual_fc1.weight.detach(), fc1_b=_param(predictor.residual_fc1, "bias"),
                 fc2_w=predictor.residual_fc2.weight.detach(), fc2_b=_param(predictor.residual_fc2, "bias"),
                 ln_w=_param(predictor.layer_norm, "weight"), ln_b=_param(predictor.layer_norm, "bias"))
        return p, KIND_RESIDUAL, float(predictor.layer_norm.eps)
    return p, KIND_FACTORIZED, 1e-5


def params_from_state_dict(state: dict, kind: str, mean=None, std=None) -> tuple[dict, int]:
    """(weights, kind code) of a predictor ``state_dict`` as the reference's checkpoints store it.

    kind is the reference's architecture name (predictor/models.py:58):
    "residual_factorized" or "factorized"; keys follow the module attributes
    (``encoder.weight``, ``residual_fc1.weight`` ...).  mean / std are folded
    into the encoder as in ``predictor_params``.
    """
    if kind not in ("residual_factorized", "factorized"):
        raise ValueError(f"Unknown predictor architecture: {kind}")

    def get(name):
        t = state.get(name)
        return None if t is None else t.detach()

    enc_w = get("encoder.weight").float()
    enc_b = get("encoder.bias")
    enc_b = None if enc_b is None else enc_b.float()
    if std is not None:
        enc_w = enc_w / std.detach().float().clamp_min(1e-6)[None, :]
    if mean is not None:
        shift = -(enc_w @ mean.detach().float())
        enc_b = shift if enc_b is None else enc_b + shift
    p = {"enc_w": enc_w, "enc_b": enc_b, "out_w": get("neurons.weight"), "out_b": get("neurons.bias")}
    if kind == "factorized":
        return p, KIND_FACTORIZED
    p.update(fc1_w=get("residual_fc1.weight"), fc1_b=get("residual_fc1.bias"), fc2_w=get("residual_fc2.weight"),
             fc2_b=get("residual_fc2.bias"), ln_w=get("layer_norm.weight"), ln_b=get("layer_norm.bias"))
    return p, KIND_RESIDUAL


class FusedScoreSelector:
    """Device copy of one predictor plus the fused scores + top-K launch."""

    def __init__(self, params: dict, *, kind: int = KIND_RESIDUAL, k: int, eps: float = 1e-5,
                 dtype: torch.dtype = torch.float32, device: torch.device | str = "cuda"):
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("qcc_b200 runs on CUDA tensors only (no CPU fallback)")
        self.code = _lib.dtype_code(dtype)
        self.dtype = dtype
        self.kind = kind
        self.eps = float(eps)
        names = ["enc_w", "enc_b", "out_w", "out_b"]
        if kind == KIND_RESIDUAL:
            names += ["fc1_w", "fc1_b", "fc2_w", "fc2_b", "ln_w", "ln_b"]
        self.w = {}
        for name in names:
            t = params.get(name)
            self.w[name] = None if t is None else t.detach().to(device=device, dtype=dtype).contiguous()
        self.latent, self.hidden = self.w["enc_w"].shape
        self.n_out = self.w["out_w"].shape[0]
        if self.w["out_w"].shape[1] != self.latent:
            raise ValueError("neuron head must take the encoder's latent width")
        if not 1 <= self.latent <= _MAX_LATENT:
            raise ValueError(f"latent width {self.latent} outside 1..{_MAX_LATENT}")
        if not 1 <= k <= self.n_out:
            raise ValueError(f"k={k} outside 1..{self.n_out}")
        self.k = k
        self.device = device
        self._lock = threading.Lock()
        self._ws = None
        self._ws_rows = 0

    @property
    def intermediate(self) -> int:
        return self.n_out

    def _workspace(self, rows: int, stream: torch.cuda.Stream) -> torch.Tensor:
        rows = min(rows, 32)
        if self._ws is None or rows > self._ws_rows:
            with self._lock:
                if self._ws is None or rows > self._ws_rows:
                    lib = _lib.library()
                    nbytes = int(lib.qcc_selector_workspace_bytes(rows, self.hidden, self.latent, self.n_out))
                    if nbytes == 0:
                        raise ValueError("qcc_selector_workspace_bytes rejected the shapes")
                    ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
                    _lib.check(lib.qcc_workspace_init(ws.data_ptr(), nbytes, stream.cuda_stream), "qcc_workspace_init")
                    self._ws, self._ws_rows = ws, rows
        return self._ws

    def check(self) -> None:
        """Raise if a call flagged a device-side timeout since the last check (synchronises)."""
        if self._ws is None:
            return
        word = self._ws[:4]
        bits = int(word.view(torch.int32).item())
        if bits:
            word.zero_()
            if bits & _lib.DEV_TIMEOUT:
                raise RuntimeError("qcc_selector_scores_topk: a bounded wait ran out (workspace re-initialised)")

    def run(self, x: torch.Tensor, *, want_scores: bool = True, k: int | None = None):
        """(scores fp32 [B, N] or None, ids int32 [B, k]) for x [B, H] (or [H])."""
        squeeze = x.dim() == 1
        if squeeze:
            x = x.unsqueeze(0)
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError(f"selector input must have shape [batch, {self.hidden}], got {tuple(x.shape)}")
        _lib.require_cuda(x)
        k = self.k if k is None else k
        if not 1 <= k <= self.n_out:
            raise ValueError(f"k={k} outside 1..{self.n_out}")
        x = x.to(self.dtype)
        if x.stride(1) != 1:
            x = x.contiguous()
        batch = x.shape[0]
        ids = torch.empty((batch, k), dtype=torch.int32, device=x.device)
        scores = torch.empty((batch, self.n_out), dtype=torch.float32, device=x.device) if want_scores else None
        stream = torch.cuda.current_stream(x.device)
        ws = self._workspace(batch, stream)
        w = self.w
        p = _lib.ptr
        lib = _lib.library()
        _lib.check(lib.qcc_selector_scores_topk(
            x.data_ptr(), x.stride(0), batch, self.hidden, self.latent, self.n_out, self.kind, self.code,
            p(w["enc_w"]), p(w["enc_b"]), p(w.get("fc1_w")), p(w.get("fc1_b")), p(w.get("fc2_w")), p(w.get("fc2_b")),
            p(w.get("ln_w")), p(w.get("ln_b")), self.eps, p(w["out_w"]), p(w["out_b"]), k, ids.data_ptr(), k,
            p(scores), self.n_out, ws.data_ptr(), ws.numel(), stream.cuda_stream), "qcc_selector_scores_topk")
        if squeeze:
            return (None if scores is None else scores[0]), ids[0]
        return scores, ids

    def scores(self, x: torch.Tensor) -> torch.Tensor:
        return self.run(x)[0]

    def select(self, x: torch.Tensor) -> torch.Tensor:
        return self.run(x, want_scores=False)[1]


class CudaSelector:
    """Drop-in for reference runtime/cuda_selector.py:45-51.

    ``folded_selector.predictor`` is a folded residual predictor (its encoder
    carries the normalisation bias); k = out_features // 2 as in the
    reference.  The reference requires fp16 weights and rounds z and the
    scores to fp16; here the predictor's dtype is kept and the arithmetic is
    fp32, scores are returned in fp32.
    """

    def __init__(self, folded_selector, device: torch.device | str | None = None):
        self.source = folded_selector
        predictor = folded_selector.predictor
        self.k = predictor.neurons.out_features // 2
        params, kind, eps = predictor_params(predictor)
        dtype = predictor.neurons.weight.dtype
        device = torch.device(device) if device is not None else predictor.neurons.weight.device
        if device.type != "cuda":
            device = torch.device("cuda", torch.cuda.current_device())
        self.engine = FusedScoreSelector(params, kind=kind, k=self.k, eps=eps, dtype=dtype, device=device)

    def scores(self, x: torch.Tensor) -> torch.Tensor:
        if x.ndim != 2 or x.shape[0] < 1:
            raise ValueError("selector input must have shape [batch, hidden] with batch >= 1")
        return self.engine.scores(x)

    def select(self, x: torch.Tensor) -> torch.Tensor:
        return self.engine.select(x)


class RuntimeSelector:
    """Drop-in for reference runtime/selector.py:15-24 (and its folded variants).

    Normalisation (mean / std) is folded into the encoder on construction
    (runtime/selector.py:31-35); ``select`` keeps ``retention_count(N,
    retention)`` neurons.  ``dtype`` is the inference dtype of the weights.
    """

    def __init__(self, predictor, mean=None, std=None, retention: float = .5, dtype: torch.dtype = torch.float32,
                 device: torch.device | str = "cuda"):
        params, kind, eps = predictor_params(predictor, mean, std)
        self.retention = retention
        k = retention_count(predictor.neurons.out_features, retention)
        self.engine = FusedScoreSelector(params, kind=kind, k=k, eps=eps, dtype=dtype, device=device)

    def scores(self, x: torch.Tensor) -> torch.Tensor:
        return self.engine.scores(x)

    def select(self, x: torch.Tensor) -> torch.Tensor:
        return self.engine.select(x)
