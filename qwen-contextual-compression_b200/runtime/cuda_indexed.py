"""Drop-in for reference runtime/cuda_indexed.py (same names and arguments).

``cuda_indexed_ffn(x, selected_ids, gate, up, down, transposed_down=False,
variant=...)`` and ``cuda_indexed_parts`` keep the reference signatures
(runtime/cuda_indexed.py:56-64) but run one fused sm_100a kernel over
neuron-major packed records.  The packed copy of (gate, up, down) is built on
first use and cached per weight tensors (invalidated when any of them is
modified in place).  ``variant`` is accepted for compatibility and ignored:
there is one kernel.  Ids may be int64 (reference contract) or int32.
"""
from __future__ import annotations

import threading
from collections import OrderedDict

import torch

from .. import _lib
from .engine import IndexedSparseFFN
from .packing import pack_neuron_major

# Accepted names; all map to the single fused kernel.
VARIANTS = {"reference": 0, "warp8": 1, "fused": 2}

_cache_lock = threading.Lock()
_engines: "OrderedDict[tuple, IndexedSparseFFN]" = OrderedDict()
_MAX_CACHED = 4


def cuda_build_diagnostic() -> dict:
    """Availability report in the shape of runtime/cuda_indexed.py:35-39."""
    if not _lib.library_path().exists():
        return {"available": False, "reason": f"qcc_b200 library not built at {_lib.library_path()}"}
    if not torch.cuda.is_available():
        return {"available": False, "reason": "PyTorch CUDA unavailable"}
    return {"available": True, "library": str(_lib.library_path())}


def load_cuda_indexed(verbose: bool = False):
    """(library, diagnostic); library is None when unavailable (runtime/cuda_indexed.py:41-49)."""
    diagnostic = cuda_build_diagnostic()
    if not diagnostic["available"]:
        return None, diagnostic
    return _lib.library(), diagnostic


def validate_selected_ids(ids: torch.Tensor, intermediate: int, expected_k: int | None = None,
                          check_bounds: bool = False) -> None:
    """Reference runtime/cuda_indexed.py:51-54, also accepting int32 ids."""
    if ids.dtype not in (torch.int64, torch.int32) or ids.ndim != 1 or not ids.is_contiguous():
        raise ValueError("selected IDs must be contiguous one-dimensional int64 or int32")
    if expected_k is not None and ids.numel() != expected_k:
        raise ValueError(f"expected {expected_k} selected IDs, got {ids.numel()}")
    if check_bounds and ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= intermediate):
        raise ValueError("selected ID out of range")


def _engine_for(gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, transposed_down: bool) -> IndexedSparseFFN:
    key = tuple((t.data_ptr(), tuple(t.shape), tuple(t.stride()), t.dtype, str(t.device), t._version)
                for t in (gate, up, down)) + (bool(transposed_down),)
    with _cache_lock:
        engine = _engines.get(key)
        if engine is not None:
            _engines.move_to_end(key)
            return engine
    engine = IndexedSparseFFN(pack_neuron_major(gate, up, down, transposed_down))
    with _cache_lock:
        _engines[key] = engine
        while len(_engines) > _MAX_CACHED:
            _engines.popitem(last=False)
    return engine


def _prepare(x, selected_ids, gate, up, down, transposed_down, variant):
    library, diagnostic = load_cuda_indexed()
    if library is None:
        raise RuntimeError(diagnostic["reason"])
    if variant not in VARIANTS:
        raise ValueError(f"Unknown CUDA indexed variant: {variant}")
    validate_selected_ids(selected_ids, gate.shape[0])
    _lib.require_cuda(x, selected_ids, gate, up, down)
    if x.dtype != gate.dtype:
        raise RuntimeError(f"x dtype {x.dtype} must match the weight dtype {gate.dtype}")
    return _engine_for(gate, up, down, transposed_down)


def cuda_indexed_ffn(x, selected_ids, gate, up, down, transposed_down=False, variant="reference"):
    """y [B, H] in x dtype (reference runtime/cuda_indexed.py:61-64)."""
    engine = _prepare(x, selected_ids, gate, up, down, transposed_down, variant)
    return engine(x, selected_ids)


def cuda_indexed_parts(x, selected_ids, gate, up, down, transposed_down=False, variant="reference"):
    """(activation, y): activation [K] (batch 1) or [B, K] in x dtype (runtime/cuda_indexed.py:56-59)."""
    engine = _prepare(x, selected_ids, gate, up, down, transposed_down, variant)
    x2 = x if x.ndim == 2 else x.unsqueeze(0)
    activation = torch.empty((x2.shape[0], selected_ids.numel()), dtype=x.dtype, device=x.device)
    y = engine(x2, selected_ids, activation=activation)
    if x.ndim == 1:
        y = y.squeeze(0)
    return (activation.squeeze(0) if x2.shape[0] == 1 else activation), y
