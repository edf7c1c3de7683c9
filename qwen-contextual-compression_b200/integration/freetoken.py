"""The engine behind the FreeToken bridge's ``runtime_factory``.

The reference routes FreeToken's layer-0 dense MLP decode rows ([1, 5120])
through ``FreeTokenQCCBridge.forward`` (integration/freetoken_qcc/bridge.py:
212-257), which builds its runtime lazily and once, under a lock, as
``runtime_factory(config)`` (bridge.py:179-205) and then calls
``runtime.run(x) -> (y, selected_ids)`` per decode row.  Its default factory,
``LazyQCCRuntime`` (bridge.py:93-176), loads fp16 safetensors weights, a
frozen predictor checkpoint folded for inference, and runs the inline CUDA
selector, ``torch.topk`` and the two-kernel indexed FFN.

``QCCBridgeRuntime`` keeps that contract (constructor taking the bridge's
config, ``initialize(device)`` once under a lock with the same device check,
``run(x) -> (y, ids)`` with y in x's dtype, the ``memory`` report) and runs
the fused score producer + top-K launch (``qcc_selector_scores_topk``) and
the fused decode over packed records.  ``runtime_weights`` may be the
reference's safetensors file (gate_proj / up_proj / down_proj.weight, packed
on the GPU at initialisation) or a packed-record artefact directory
(``runtime.artefact``), loaded as is.  Pass ``QCCBridgeRuntime`` (or
``make_runtime_factory(...)``) as the bridge's ``runtime_factory``.

Differences kept on purpose: the ids come back as ascending int32 (the
reference's ``torch.topk(sorted=False)`` order is unspecified and int64), the
selector's arithmetic is fp32 on the checkpoint's weights cast to the layer's
dtype (the reference rounds its latent and scores to fp16), and weights may be
fp16, bf16 or fp32.
"""
from __future__ import annotations

import json
import threading
from pathlib import Path

import torch

from ..runtime import artefact
from ..runtime.cuda_indexed import VARIANTS
from ..runtime.cuda_selector import FusedScoreSelector, params_from_state_dict, retention_count
from ..runtime.engine import IndexedSparseFFN
from ..runtime.packing import pack_neuron_major, validate_weight_shapes

EXPECTED_HIDDEN = 5120        # integration/freetoken_qcc/bridge.py:19
EXPECTED_INTERMEDIATE = 17408  # integration/freetoken_qcc/bridge.py:20
LAYER_NORM_EPS = 1e-5          # nn.LayerNorm default of the reference's predictor


def load_selector_checkpoint(path: Path | str, retention: float, device: torch.device,
                             dtype: torch.dtype) -> tuple[FusedScoreSelector, dict]:
    """Fused selector from a reference predictor checkpoint (runtime/selector.py:19-20 format).

    The checkpoint holds ``config`` (kind, input_dim, output_dim, latent_dim),
    ``model`` (the predictor's state_dict), ``mean`` and ``std``; the
    normalisation is folded into the encoder (runtime/selector.py:31-35).
    """
    checkpoint = torch.load(str(path), map_location="cpu", weights_only=True)
    config = checkpoint["config"]
    params, kind = params_from_state_dict(checkpoint["model"], config["kind"], checkpoint["mean"].float(),
                                          checkpoint["std"].float())
    if params["enc_w"].shape != (config["latent_dim"], config["input_dim"]):
        raise ValueError("Selector checkpoint encoder does not match its config")
    k = retention_count(config["output_dim"], retention)
    selector = FusedScoreSelector(params, kind=kind, k=k, eps=LAYER_NORM_EPS, dtype=dtype, device=device)
    return selector, config


class QCCBridgeRuntime:
    """Drop-in for the bridge's ``LazyQCCRuntime``: lazily initialised selector + fused decode."""

    def __init__(self, config, *, expected_shape: tuple[int, int] | None = None):
        self.config = config
        self.expected_shape = tuple(expected_shape) if expected_shape else (EXPECTED_HIDDEN, EXPECTED_INTERMEDIATE)
        self.device = None
        self.memory: dict = {}
        self.initialized = False
        self._initialize_lock = threading.Lock()
        self.engine: IndexedSparseFFN | None = None
        self.selector: FusedScoreSelector | None = None

    def initialize(self, device: torch.device) -> None:
        if self.initialized:
            if self.device != device:
                raise RuntimeError(f"QCC runtime initialized on {self.device}, but received input on {device}")
            return
        with self._initialize_lock:
            if self.initialized:
                if self.device != device:
                    raise RuntimeError(f"QCC runtime initialized on {self.device}, but received input on {device}")
                return
            self._initialize(device)

    def _load_weights(self, device: torch.device):
        path = Path(self.config.runtime_weights)
        if path.is_dir():
            weights = artefact.load_packed_layer(path, device, expected_shape=self.expected_shape)
            return weights, artefact.load_manifest(path).get("metadata", {})
        from safetensors import safe_open
        from safetensors.torch import load_file

        tensors = load_file(str(path), device=str(device))
        missing = [role for role in artefact.ROLES if role not in tensors]
        if missing:
            raise ValueError(f"QCC runtime weights are missing {missing}")
        gate, up, down = (tensors[role] for role in artefact.ROLES)
        hidden, intermediate = validate_weight_shapes(gate, up, down)
        if (hidden, intermediate) != self.expected_shape:
            raise ValueError(f"QCC runtime weights are {(hidden, intermediate)}, expected {self.expected_shape}")
        weights = pack_neuron_major(gate, up, down)
        del tensors, gate, up, down
        with safe_open(str(path), framework="pt", device="cpu") as handle:
            metadata = handle.metadata() or {}
        return weights, metadata

    def _initialize(self, device: torch.device) -> None:
        if device.type != "cuda":
            raise RuntimeError("QCC FreeToken replacement requires a CUDA input tensor")
        if self.config.variant not in VARIANTS:
            raise ValueError(f"Unknown CUDA indexed variant: {self.config.variant}")
        allocated_before = torch.cuda.memory_allocated(device)
        reserved_before = torch.cuda.memory_reserved(device)
        weights, metadata = self._load_weights(device)
        hidden, intermediate = weights.hidden, weights.n_records
        selector, sel_config = load_selector_checkpoint(self.config.selector_checkpoint, self.config.retention,
                                                        device, weights.dtype)
        if selector.hidden != hidden or selector.n_out != intermediate:
            raise ValueError(f"Selector dimensions {(selector.hidden, selector.n_out)} do not match the layer "
                             f"{(hidden, intermediate)}")
        self.engine = IndexedSparseFFN(weights)
        self.selector = selector
        self.device = device
        self.initialized = True
        allocated_after = torch.cuda.memory_allocated(device)
        reserved_after = torch.cuda.memory_reserved(device)
        selector_bytes = sum(t.numel() * t.element_size() for t in selector.w.values() if t is not None)
        self.memory = {
            "allocated_before": allocated_before,
            "allocated_after": allocated_after,
            "reserved_before": reserved_before,
            "reserved_after": reserved_after,
            "qcc_added_allocated_mib": (allocated_after - allocated_before) / 2**20,
            "ffn_weight_bytes": weights.packed.numel() * weights.packed.element_size(),
            "selector_bytes": selector_bytes,
            "selector": {"kind": sel_config["kind"], "latent_dim": sel_config["latent_dim"], "k": selector.k},
            "metadata": metadata,
            "layout": "neuron-major packed records",
        }
        print("QCC FreeToken lazy initialization: " + json.dumps(self.memory, default=str, sort_keys=True))

    @torch.inference_mode()
    def run(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(y in x's dtype, ascending int32 selected ids) for one decode row x [1, hidden]."""
        self.initialize(x.device)
        xw = x.to(dtype=self.engine.weights.dtype).contiguous()
        selected_ids = self.selector.select(xw)[0]
        y = self.engine(xw, selected_ids)
        return y.to(dtype=x.dtype), selected_ids

    def check(self) -> None:
        """Raise if a call flagged a device-side error (synchronises)."""
        if self.initialized:
            self.selector.check()
            self.engine.check()


def make_runtime_factory(**options):
    """A ``runtime_factory`` for the bridge that passes ``options`` (e.g. ``expected_shape``) on."""
    def factory(config):
        return QCCBridgeRuntime(config, **options)
    return factory


runtime_factory = QCCBridgeRuntime
