"""Host-side mirror of the reference's ``runtime`` package for the hot path."""
from .packing import PackedFFNWeights, pack_neuron_major, validate_weight_shapes  # noqa: F401
from .engine import IndexedSparseFFN  # noqa: F401
from .cuda_indexed import cuda_indexed_ffn, cuda_indexed_parts, validate_selected_ids  # noqa: F401
from .triton_sparse_ffn import triton_indexed_ffn  # noqa: F401
from .ffn import TorchDynamicSparseFFN  # noqa: F401
from .selector import TopKSelector, build_union, retention_count, select_topk  # noqa: F401
