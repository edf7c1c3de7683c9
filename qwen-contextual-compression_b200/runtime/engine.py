"""The fused indexed gated-FFN engine (one packed layer on one GPU).

``IndexedSparseFFN(weights)(x, ids)`` computes, in one kernel launch per
chunk of <= 4 tokens,

    y[b] = sum_j mask[j, b] * silu(G[ids_j] . x[b]) * (U[ids_j] . x[b]) * D[:, ids_j]

which is reference runtime/ffn.py:34-39 (``TorchDynamicSparseFFN.forward``)
and runtime/cuda_indexed.py:61-64 (``cuda_indexed_ffn``) without gathered
copies.  The fp32 accumulation workspace is owned here, one per CUDA stream,
zeroed once; the kernel leaves it zeroed after every call.
"""
from __future__ import annotations

import threading

import torch

from .. import _lib
from .packing import PackedFFNWeights


class DecodeWorkspace:
    """Zero-initialised scratch for qcc_indexed_ffn_decode on one stream."""

    def __init__(self, device: torch.device, batch: int, hidden: int, dtype: torch.dtype, stream: torch.cuda.Stream):
        lib = _lib.library()
        code = _lib.dtype_code(dtype)
        self.nbytes = int(lib.qcc_decode_workspace_bytes(batch, hidden, code))
        if self.nbytes == 0:
            raise ValueError(f"no decode workspace for batch={batch} hidden={hidden}")
        self.buffer = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.status_offset = int(lib.qcc_workspace_status_offset())
        _lib.check(lib.qcc_workspace_init(self.buffer.data_ptr(), self.nbytes, stream.cuda_stream),
                   "qcc_workspace_init")

    def read_status(self, clear: bool = True) -> int:
        """Device status bits (synchronises with the buffer's stream)."""
        word = self.buffer[self.status_offset:self.status_offset + 4]
        value = int(word.view(torch.int32).item())
        if clear and value:
            word.zero_()
        return value


class IndexedSparseFFN:
    """Fused indexed sparse FFN over neuron-major packed records.

    ``check_bounds=True`` reads the device status after every call (a host
    sync) and raises ``ValueError("selected ID out of range")`` like reference
    runtime/cuda_indexed.py:51-54; otherwise out-of-range ids contribute
    nothing and are reported by :meth:`check`.
    """

    def __init__(self, weights: PackedFFNWeights, check_bounds: bool = False):
        self.weights = weights
        self.check_bounds = check_bounds
        lib = _lib.library()
        self._code = _lib.dtype_code(weights.dtype)
        self.max_batch = int(lib.qcc_decode_max_batch(weights.hidden, self._code))
        if self.max_batch < 1:
            raise ValueError(f"hidden={weights.hidden} is beyond the decode kernel's limit")
        self._workspaces: dict[int, DecodeWorkspace] = {}
        self._lock = threading.Lock()

    @property
    def hidden(self) -> int:
        return self.weights.hidden

    @property
    def intermediate(self) -> int:
        return self.weights.n_records

    def workspace(self, stream: torch.cuda.Stream) -> DecodeWorkspace:
        key = stream.cuda_stream
        ws = self._workspaces.get(key)
        if ws is None:
            with self._lock:
                ws = self._workspaces.get(key)
                if ws is None:
                    ws = DecodeWorkspace(self.weights.device, self.max_batch, self.hidden, self.weights.dtype, stream)
                    self._workspaces[key] = ws
        return ws

    def check(self) -> None:
        """Raise if any call since the last check flagged a device-side error."""
        for ws in list(self._workspaces.values()):
            bits = ws.read_status()
            if bits & _lib.DEV_ID_RANGE:
                raise ValueError("selected ID out of range")
            if bits & _lib.DEV_TIMEOUT:
                raise RuntimeError("qcc_indexed_ffn_decode: a bounded wait on a bulk copy ran out")

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, **kwargs) -> torch.Tensor:
        return self.forward(x, ids, **kwargs)

    def forward(self, x: torch.Tensor, ids: torch.Tensor, *, token_mask: torch.Tensor | None = None,
                n_ids_dev: torch.Tensor | None = None, out: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None, activation: torch.Tensor | None = None) -> torch.Tensor:
        """y [B, H] for x [B, H] (or [H] -> [H]) and the 1-D selected-id list ``ids``.

        token_mask: optional uint8 [len(ids)], bit b = token b uses record j.
        n_ids_dev:  optional int32 device scalar; only the first n ids are used.
        out_dtype:  x.dtype (default) or torch.float32 (unrounded partial sums).
        activation: optional [B, len(ids)] tensor in x.dtype receiving a_j.
        """
        w = self.weights
        squeeze = x.ndim == 1
        if squeeze:
            x = x.unsqueeze(0)
        if x.ndim != 2 or x.shape[1] != w.hidden:
            raise ValueError(f"x must be [batch, {w.hidden}], got {tuple(x.shape)}")
        if x.dtype != w.dtype:
            raise TypeError(f"x dtype {x.dtype} must match the weight dtype {w.dtype}")
        if ids.ndim != 1 or not ids.is_contiguous():
            raise ValueError("selected IDs must be contiguous one-dimensional int32 or int64")
        if ids.dtype not in _lib.INDEX_DTYPES:
            raise ValueError("selected IDs must be contiguous one-dimensional int32 or int64")
        device = _lib.require_cuda(x, ids, w.packed, token_mask, n_ids_dev, out, activation)
        if x.stride(1) != 1:
            x = x.contiguous()
        batch = x.shape[0]
        n_ids = ids.numel()
        if token_mask is not None and (token_mask.dtype != torch.uint8 or token_mask.numel() < n_ids
                                       or not token_mask.is_contiguous()):
            raise ValueError("token_mask must be a contiguous uint8 tensor with one byte per id")
        if n_ids_dev is not None and (n_ids_dev.dtype != torch.int32 or n_ids_dev.numel() != 1):
            raise ValueError("n_ids_dev must be a one-element int32 tensor")
        out_dtype = out_dtype or x.dtype
        if out is None:
            out = torch.empty((batch, w.hidden), dtype=out_dtype, device=device)
        elif out.shape != (batch, w.hidden) or out.stride(1) != 1 or out.dtype != out_dtype:
            raise ValueError("out must be a row-contiguous [batch, hidden] tensor of out_dtype")
        if activation is not None and (activation.shape != (batch, n_ids) or activation.dtype != x.dtype
                                       or activation.stride(1) != 1):
            raise ValueError("activation must be a row-contiguous [batch, n_ids] tensor in x dtype")
        lib = _lib.library()
        stream = torch.cuda.current_stream(device)
        ws = self.workspace(stream)
        y_code = _lib.dtype_code(out_dtype)
        esize_x, esize_y = x.element_size(), out.element_size()
        for start in range(0, batch, self.max_batch):
            chunk = min(self.max_batch, batch - start)
            a_ptr = None if activation is None else activation.data_ptr() + start * activation.stride(0) * esize_x
            mask = token_mask
            if mask is not None and start > 0:
                # Token bits start.. moved down to bit 0.  The temporary comes from
                # the caching allocator on this stream, so its reuse is ordered
                # after the kernel that reads it.
                mask = torch.bitwise_right_shift(token_mask, start)
            status = lib.qcc_indexed_ffn_decode(
                x.data_ptr() + start * x.stride(0) * esize_x, x.stride(0), chunk, w.hidden, w.packed.data_ptr(),
                w.n_records, self._code, ids.data_ptr(), _lib.INDEX_DTYPES[ids.dtype], n_ids,
                _lib.ptr(n_ids_dev), _lib.ptr(mask), ws.buffer.data_ptr(), ws.nbytes,
                out.data_ptr() + start * out.stride(0) * esize_y, out.stride(0), y_code, a_ptr,
                n_ids if activation is not None else 0, stream.cuda_stream)
            _lib.check(status, "qcc_indexed_ffn_decode")
        if self.check_bounds:
            self.check()
        return out.squeeze(0) if squeeze else out
