"""qcc_b200 -- B200-native indexed sparse gated-FFN engine.

The contextual-sparsity hot path of robjlyons/qwen-contextual-compression
(per-neuron scores -> top-K selection -> fused indexed gated FFN), rebuilt as
hand-written sm_100a CUDA behind a C ABI (``include/qcc_b200.h``,
``libqcc_b200.so``) with a host API that mirrors the reference's Python call
surface:

* ``qcc_b200.runtime.cuda_indexed``  -- ``cuda_indexed_ffn``, ``cuda_indexed_parts``,
  ``validate_selected_ids`` (reference runtime/cuda_indexed.py)
* ``qcc_b200.runtime.ffn``           -- ``TorchDynamicSparseFFN`` (reference runtime/ffn.py)
* ``qcc_b200.runtime.selector``      -- deterministic top-K selection (reference runtime/selector.py)
* ``qcc_b200.runtime.sharded``       -- intermediate-dimension sharding over GPUs
* ``qcc_b200.end_to_end``            -- ``OracleSparseMLP``, ``OracleMLPPatcher``

There is no CPU fallback: every compute entry point raises if the CUDA
library is missing or the tensors are not on a CUDA device.
"""
from __future__ import annotations

__version__ = "0.1.0"

from . import _lib  # noqa: F401  (library binding; loads lazily)
from ._lib import QCCError, library_path  # noqa: F401
