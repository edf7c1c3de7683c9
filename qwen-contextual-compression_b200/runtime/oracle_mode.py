"""Oracle-mode FFN over packed records: dense gate/up, selection by the live activation, indexed down.

The reference's oracle keeps, per token, the K neurons whose activation
matters most and drops the rest: importance |a| or |a| * ||D[:, j]||_2
(oracle/importance.py:6-13), top K (oracle/importance.py:21-23), then
y = D[:, ids] a[ids] (oracle/sparse_ffn.py:8-13); ``OracleSparseMLP`` does
the same inside a model with |a| * ||D[:, j]||, ``torch.topk``, a scatter into
zeros and a dense down projection (end_to_end/oracle_sparse_mlp.py:64-78).
Gate and up are dense by construction: the selection needs every neuron's
activation.

Here one layer is three kinds of launch per chunk of tokens:

1. ``qcc_ffn_activations`` streams the gate | up part of every record (2/3 of
   the layer) and writes the fp32 activation of every neuron;
2. ``qcc_activation_topk`` scores each token's activations (|a| or |a| * w)
   and selects its K neurons, one CTA per token;
3. ``qcc_indexed_ffn_down`` streams only the down part of the union of the
   tokens' selections (per-token bits from ``qcc_build_union``) and sums
   y = sum_j a_j D_j in a fixed order.

So a token reads 2/3 of the layer plus K/N of the last third, instead of the
whole layer twice over as the masked-dense formulation does.
"""
from __future__ import annotations

import torch

from .. import _lib
from .engine import _current_stream, stream_workspace
from .packing import PackedFFNWeights
from .selector import activation_topk, build_union, retention_count

SCORES = ("activation", "weighted_activation")


def down_column_norms(weights: PackedFFNWeights) -> torch.Tensor:
    """fp32 ||D[:, j]||_2 of every record's down part (the weights of the "weighted_activation" score).

    Sums of squares in float64, rounded once, so the result is within half an
    fp32 ulp of the exact norm (one-time preparation on the records' device).
    """
    hp = weights.hidden_pad
    down = weights.packed[:, 2 * hp:2 * hp + weights.hidden]
    return down.double().square().sum(dim=1).sqrt().float().contiguous()


class OracleModeFFN:
    """``(y, ids) = OracleModeFFN(weights, retention)(x)`` for x [T, hidden]."""

    def __init__(self, weights: PackedFFNWeights, retention: float, score: str = "weighted_activation",
                 column_weights: torch.Tensor | None = None):
        if score not in SCORES:
            raise ValueError(f"score must be one of {SCORES}")
        self.weights = weights
        self.retention = float(retention)
        self.k = retention_count(weights.n_records, retention)
        self.score = score
        lib = _lib.library()
        self._code = _lib.dtype_code(weights.dtype)
        self.max_batch = int(lib.qcc_decode_max_batch(weights.hidden, self._code))
        if self.max_batch < 1:
            raise ValueError(f"hidden={weights.hidden} is beyond the decode kernels' limit")
        self._ws_bytes = int(lib.qcc_decode_workspace_bytes(self.max_batch, weights.hidden, self._code))
        if score == "weighted_activation":
            w = column_weights if column_weights is not None else down_column_norms(weights)
            self.column_weights = w.to(device=weights.device, dtype=torch.float32).contiguous()
        else:
            self.column_weights = None

    def activations(self, x: torch.Tensor) -> torch.Tensor:
        """fp32 [T, N] silu(G x) * (U x) of every record, from the gate | up parts only."""
        w = self.weights
        if x.ndim != 2 or x.shape[1] != w.hidden or x.dtype != w.dtype:
            raise ValueError(f"x must be [tokens, {w.hidden}] in {w.dtype}")
        _lib.require_cuda(x, w.packed)
        x = x.contiguous()
        n = w.n_records
        acts = torch.empty((x.shape[0], n), dtype=torch.float32, device=x.device)
        stream = _current_stream(x.device.index)
        ws = stream_workspace(x.device, torch.cuda.current_stream(x.device), self._ws_bytes)
        lib = _lib.library()
        for start in range(0, x.shape[0], self.max_batch):
            rows = min(self.max_batch, x.shape[0] - start)
            _lib.check(lib.qcc_ffn_activations(x[start].data_ptr(), x.stride(0), rows, w.hidden, w.packed.data_ptr(), n,
                                               self._code, None, acts[start].data_ptr(), n, None, 0, ws.ptr,
                                               ws.nbytes, stream), "qcc_ffn_activations")
        return acts

    def select(self, acts: torch.Tensor) -> torch.Tensor:
        """Ascending int32 ids [T, K] of each token's K most important neurons."""
        return activation_topk(acts, self.k, self.column_weights)

    def down(self, acts: torch.Tensor, ids: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """y [T, hidden]: the down parts of each token's selected records weighted by its activations."""
        w = self.weights
        tokens = acts.shape[0]
        out_dtype = out_dtype or w.dtype
        y = torch.empty((tokens, w.hidden), dtype=out_dtype, device=acts.device)
        stream = _current_stream(acts.device.index)
        ws = stream_workspace(acts.device, torch.cuda.current_stream(acts.device), self._ws_bytes)
        lib = _lib.library()
        for start in range(0, tokens, self.max_batch):
            rows = min(self.max_batch, tokens - start)
            union, mask, count = build_union(ids[start:start + rows], 0, w.n_records)
            _lib.check(lib.qcc_indexed_ffn_down(
                acts[start].data_ptr(), acts.stride(0), _lib.DTYPE_F32, rows, w.hidden, w.packed.data_ptr(),
                w.n_records, self._code, union.data_ptr(), _lib.INDEX_I32, union.numel(), count.data_ptr(),
                mask.data_ptr(), ws.ptr, ws.nbytes, y[start].data_ptr(), y.stride(0), _lib.dtype_code(out_dtype),
                None, 0, stream), "qcc_indexed_ffn_down")
        return y

    def __call__(self, x: torch.Tensor, out_dtype: torch.dtype | None = None):
        return self.forward(x, out_dtype)

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype | None = None):
        """(y [T, hidden], ids [T, K]) for x [T, hidden] (or [hidden])."""
        squeeze = x.ndim == 1
        if squeeze:
            x = x.unsqueeze(0)
        acts = self.activations(x)
        ids = self.select(acts)
        y = self.down(acts, ids, out_dtype)
        return (y[0], ids[0]) if squeeze else (y, ids)

    def check(self) -> None:
        """Raise if a call flagged a device-side error (synchronises)."""
        from .engine import _workspaces
        for (dev, _), ws in list(_workspaces.items()):
            if dev == self.weights.device.index:
                bits = ws.read_status()
                if bits & _lib.DEV_TIMEOUT:
                    raise RuntimeError("oracle-mode FFN: a bounded wait on a record copy ran out")
