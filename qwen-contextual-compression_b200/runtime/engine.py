"""The fused indexed gated-FFN engine (one packed layer on one GPU).

``IndexedSparseFFN(weights)(x, ids)`` computes, in one call of the C ABI
(a record-streaming launch and a reduce launch) per chunk of up to
``max_batch`` tokens (``qcc_decode_max_batch``: 8 at hidden 5120 for 16-bit
records, whose 2-8 token chunks run on the tensor cores),

    y[b] = sum_j mask[j, b] * silu(G[ids_j] . x[b]) * (U[ids_j] . x[b]) * D[:, ids_j]

which is reference runtime/ffn.py:34-39 (``TorchDynamicSparseFFN.forward``)
and runtime/cuda_indexed.py:61-64 (``cuda_indexed_ffn``) without gathered
copies.  The kernel's scratch (a status word, a counter and one fp32
partial-y row per CTA) is a device buffer shared by every engine that
launches on the same CUDA stream -- launches on one stream never overlap --
zeroed once; the kernels leave the counter at zero after every call.
"""
from __future__ import annotations

import threading

import torch

from .. import _lib
from .packing import PackedFFNWeights


class DecodeWorkspace:
    """Zero-initialised scratch for qcc_indexed_ffn_decode on one stream."""

    def __init__(self, device: torch.device, nbytes: int, stream: torch.cuda.Stream):
        lib = _lib.library()
        self.nbytes = nbytes
        self.buffer = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.ptr = self.buffer.data_ptr()
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


_workspace_lock = threading.Lock()
_workspaces: dict[tuple[int, int], DecodeWorkspace] = {}


def stream_workspace(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> DecodeWorkspace:
    """The shared workspace of (device, stream), grown to at least nbytes."""
    key = (device.index, stream.cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.nbytes < nbytes:
        with _workspace_lock:
            ws = _workspaces.get(key)
            if ws is None or ws.nbytes < nbytes:
                old = ws
                ws = DecodeWorkspace(device, nbytes, stream)
                if old is not None:
                    status = old.read_status(clear=True)  # carry pending device errors over
                    if status:
                        ws.buffer[:4].view(torch.int32).fill_(status)
                _workspaces[key] = ws
    return ws


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
        self._workspace_bytes = int(lib.qcc_decode_workspace_bytes(self.max_batch, weights.hidden, self._code))
        self._streams: set[int] = set()
        self._streams_ws: dict[int, DecodeWorkspace] = {}
        self._plans: dict = {}

    @property
    def hidden(self) -> int:
        return self.weights.hidden

    @property
    def intermediate(self) -> int:
        return self.weights.n_records

    def workspace(self, stream: torch.cuda.Stream) -> DecodeWorkspace:
        self._streams.add(stream.cuda_stream)
        return stream_workspace(self.weights.device, stream, self._workspace_bytes)

    def check(self) -> None:
        """Raise if a call on this engine's streams flagged a device-side error since the last check."""
        for ws in list(self._streams_ws.values()):
            bits = ws.read_status()
            if bits & _lib.DEV_ID_RANGE:
                raise ValueError("selected ID out of range")
            if bits & _lib.DEV_TIMEOUT:
                raise RuntimeError("qcc_indexed_ffn_decode: a bounded wait ran out (a record copy, or the "
                                   "other ranks' sums of a cross-rank exchange)")

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, **kwargs) -> torch.Tensor:
        return self.forward(x, ids, **kwargs)

    def forward(self, x: torch.Tensor, ids: torch.Tensor, *, token_mask: torch.Tensor | None = None,
                n_ids_dev: torch.Tensor | None = None, out: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None, activation: torch.Tensor | None = None,
                accumulate: torch.Tensor | None = None, exchange=None,
                id_range: tuple[int, int] | None = None, ids_ready: bool = False) -> torch.Tensor:
        """y [B, H] for x [B, H] (or [H] -> [H]) and the 1-D selected-id list ``ids``.

        token_mask: optional uint8 [len(ids)], bit b = token b uses record j.
        n_ids_dev:  optional int32 device scalar; only the first n ids are used.
        out_dtype:  x.dtype (default) or torch.float32 (unrounded partial sums).
        activation: optional [B, len(ids)] tensor in x.dtype receiving a_j.
        accumulate: optional fp32 [B, H] added before the final rounding.
        exchange:   optional cross-rank exchange (``sharded.PeerExchange``): y is
                    then the sum of every rank's partial over this rank's shard.
        id_range:   optional (begin, end): ``ids`` is the global ascending id
                    list and only its ids in [begin, end), rebased by begin,
                    select records of this engine (the kernel finds the run).
        ids_ready:  the ids (and token_mask / n_ids_dev) were not written by an
                    earlier qcc_b200 launch on this stream (e.g. they came from
                    a host copy): the kernel then starts its record copies
                    before the launches ahead of it finish (QCC_IDS_READY).
                    Leave it False for ids from ``select_topk``,
                    ``build_union`` or the fused selector on the same stream.
        """
        squeeze = x.dim() == 1
        if squeeze:
            x = x.unsqueeze(0)
        plan = self._plan(x, ids, token_mask, n_ids_dev, out, out_dtype, activation)
        if x.stride(1) != 1:
            x = x.contiguous()
        batch = x.shape[0]
        n_ids = ids.shape[0]
        if out is None:
            out = torch.empty((batch, self.weights.hidden), dtype=plan.out_dtype, device=x.device)
        stream = _current_stream(plan.device_index)
        ws = self._streams_ws.get(stream)
        if ws is None:
            ws = self._workspace_for(stream)
        lib = plan.lib
        ids_code = plan.ids_code | (_lib.IDS_READY if ids_ready else 0)
        x_ptr, out_ptr = x.data_ptr(), out.data_ptr()
        x_row, out_row = x.stride(0) * plan.esize_x, out.stride(0) * plan.esize_y
        mask_ptr = None if token_mask is None else token_mask.data_ptr()
        count_ptr = None if n_ids_dev is None else n_ids_dev.data_ptr()
        acc_row = acc_ld = 0
        if accumulate is not None:
            if (accumulate.dtype != torch.float32 or accumulate.shape != (batch, plan.hidden)
                    or accumulate.stride(1) != 1 or accumulate.device != x.device):
                raise ValueError("accumulate must be a row-contiguous fp32 [batch, hidden] tensor on x's device")
            acc_ld = accumulate.stride(0)
            acc_row = acc_ld * 4
        for start in range(0, batch, self.max_batch):
            chunk = min(self.max_batch, batch - start)
            a_ptr = None if activation is None else activation.data_ptr() + start * activation.stride(0) * plan.esize_x
            # The chunk's tokens read bits start.. of the same mask (QCC_MASK_SHIFT).
            chunk_code = ids_code | (_lib.mask_shift(start) if token_mask is not None else 0)
            acc_ptr = None if accumulate is None else accumulate.data_ptr() + start * acc_row
            if exchange is not None or id_range is not None:
                if a_ptr is not None:
                    raise ValueError("activation output is not available with a cross-rank exchange or id range")
                id_begin, id_end = id_range if id_range is not None else (-1, -1)
                if id_range is not None and not 0 <= id_begin <= id_end:
                    raise ValueError("id_range must satisfy 0 <= begin <= end")
                world, rank = (exchange.world, exchange.rank) if exchange is not None else (1, 0)
                status = lib.qcc_indexed_ffn_decode_allreduce(
                    x_ptr + start * x_row, x.stride(0), chunk, plan.hidden, plan.packed_ptr, plan.n_records,
                    plan.code, ids.data_ptr(), chunk_code, n_ids, count_ptr, mask_ptr, ws.ptr, ws.nbytes,
                    out_ptr + start * out_row, out.stride(0), plan.y_code, acc_ptr, acc_ld, id_begin, id_end,
                    exchange.pointers if exchange is not None else None,
                    exchange.nbytes if exchange is not None else 0, world, rank, stream)
                if status:
                    _lib.check(status, "qcc_indexed_ffn_decode_allreduce")
                continue
            status = lib.qcc_indexed_ffn_decode(
                x_ptr + start * x_row, x.stride(0), chunk, plan.hidden, plan.packed_ptr, plan.n_records, plan.code,
                ids.data_ptr(), chunk_code, n_ids, count_ptr, mask_ptr, ws.ptr, ws.nbytes,
                out_ptr + start * out_row, out.stride(0), plan.y_code, acc_ptr, acc_ld, a_ptr, n_ids if a_ptr else 0,
                stream)
            if status:
                _lib.check(status, "qcc_indexed_ffn_decode")
        if self.check_bounds:
            self.check()
        return out.squeeze(0) if squeeze else out

    def _workspace_for(self, stream_handle: int) -> DecodeWorkspace:
        stream = torch.cuda.ExternalStream(stream_handle, device=self.weights.device)
        ws = self.workspace(stream)
        self._streams_ws[stream_handle] = ws
        return ws

    def _plan(self, x, ids, token_mask, n_ids_dev, out, out_dtype, activation) -> "_Plan":
        """Checks that depend only on shapes / dtypes / devices, cached per signature."""
        key = (x.shape, x.dtype, x.device, ids.dim(), ids.dtype, ids.device, ids.is_contiguous(), out_dtype,
               None if out is None else (out.shape, out.dtype, out.stride(1), out.device),
               None if token_mask is None else (token_mask.dtype, token_mask.is_contiguous(), token_mask.numel()),
               None if n_ids_dev is None else (n_ids_dev.dtype, n_ids_dev.numel(), n_ids_dev.device),
               None if activation is None else (activation.shape, activation.dtype, activation.stride(1)),
               ids.shape)
        plan = self._plans.get(key)
        if plan is not None:
            return plan
        w = self.weights
        if x.dim() != 2 or x.shape[1] != w.hidden:
            raise ValueError(f"x must be [batch, {w.hidden}], got {tuple(x.shape)}")
        if x.dtype != w.dtype:
            raise TypeError(f"x dtype {x.dtype} must match the weight dtype {w.dtype}")
        if ids.dim() != 1 or not ids.is_contiguous() or ids.dtype not in _lib.INDEX_DTYPES:
            raise ValueError("selected IDs must be contiguous one-dimensional int32 or int64")
        device = _lib.require_cuda(x, ids, w.packed, token_mask, n_ids_dev, out, activation)
        batch, n_ids = x.shape[0], ids.shape[0]
        if token_mask is not None and batch > 8:
            raise ValueError("a token_mask holds 8 tokens per byte: batch must be <= 8 with a token_mask")
        if token_mask is not None and (token_mask.dtype != torch.uint8 or token_mask.numel() < n_ids
                                       or not token_mask.is_contiguous()):
            raise ValueError("token_mask must be a contiguous uint8 tensor with one byte per id")
        if n_ids_dev is not None and (n_ids_dev.dtype != torch.int32 or n_ids_dev.numel() != 1):
            raise ValueError("n_ids_dev must be a one-element int32 tensor")
        out_dtype = out_dtype or (out.dtype if out is not None else x.dtype)
        if out is not None and (out.shape != (batch, w.hidden) or out.stride(1) != 1 or out.dtype != out_dtype):
            raise ValueError("out must be a row-contiguous [batch, hidden] tensor of out_dtype")
        if activation is not None and (activation.shape != (batch, n_ids) or activation.dtype != x.dtype
                                       or activation.stride(1) != 1):
            raise ValueError("activation must be a row-contiguous [batch, n_ids] tensor in x dtype")
        plan = _Plan(lib=_lib.library(), device_index=device.index, hidden=w.hidden, packed_ptr=w.packed.data_ptr(),
                     n_records=w.n_records, code=self._code, ids_code=_lib.INDEX_DTYPES[ids.dtype],
                     out_dtype=out_dtype, y_code=_lib.dtype_code(out_dtype), esize_x=x.element_size(),
                     esize_y=torch.empty((), dtype=out_dtype).element_size())
        if len(self._plans) > 64:
            self._plans.clear()
        self._plans[key] = plan
        return plan


class _Plan:
    __slots__ = ("lib", "device_index", "hidden", "packed_ptr", "n_records", "code", "ids_code", "out_dtype",
                 "y_code", "esize_x", "esize_y")

    def __init__(self, **kw):
        for k, v in kw.items():
            setattr(self, k, v)


def _current_stream(device_index: int) -> int:
    """Raw handle of the current CUDA stream of a device."""
    return _raw_stream(device_index)


try:  # the raw-handle query avoids building a torch.cuda.Stream object per call
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover
    def _raw_stream(device_index: int) -> int:
        return torch.cuda.current_stream(device_index).cuda_stream
