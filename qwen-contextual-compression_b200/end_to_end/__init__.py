"""Model-level drop-ins: the x-only oracle MLP wrapper and the reversible patcher."""
from .oracle_sparse_mlp import OracleSparseMLP, compute_down_column_norms_chunked  # noqa: F401
from .model_patcher import OracleMLPPatcher, find_gated_mlps  # noqa: F401
