"""Block-sparse prefill: 128-token tiles, each with its own set of 64-record blocks.

In the reference a prefill selection comes in whole blocks: block top-K
(``oracle/importance.py:26-35``) or ``select_blocks`` / ``expand_block_indices``
(``clustering/block_layout.py:22-64``) turn block ids into neuron ids, and each
tile of tokens then runs ``TorchDynamicSparseFFN`` (``runtime/ffn.py:20-39``)
on its expanded ids.  :class:`BlockSparsePrefill` takes the block ids of every
tile and runs the whole prefill as tensor-core GEMMs over the packed records
(``qcc_indexed_ffn_prefill``).  The units of a block pair shared by several
tiles run side by side and keep its rows in L2, so DRAM sees it about once.

bf16 and fp16 records run on ``tcgen05.mma kind::f16``; fp32 records run on
``kind::tf32``: the products use the tf32 part of each fp32 operand (x, the
gate / up / down rows and the intermediate activations), the sums are fp32.
"""
from __future__ import annotations

from typing import Sequence

import torch

from .. import _lib
from .packing import PackedFFNWeights

TILE_TOKENS = 128
BLOCK_RECORDS = 64


def blocks_of_ids(ids: torch.Tensor, block_size: int = BLOCK_RECORDS, n_records: int | None = None) -> torch.Tensor:
    """Block ids of a neuron-id list made of whole blocks (``expand_block_indices`` inverted).

    The last block may be partial when it ends at ``n_records``.  Raises
    ``ValueError`` if the ids are not a union of complete blocks.
    """
    if block_size != BLOCK_RECORDS:
        raise ValueError(f"expected block_size {BLOCK_RECORDS}, got {block_size}")
    ids = torch.as_tensor(ids).flatten().to(torch.int64).unique()
    blocks = torch.unique(torch.div(ids, block_size, rounding_mode="floor"))
    sizes = torch.full_like(blocks, block_size)
    if n_records is not None:
        sizes = torch.clamp(n_records - blocks * block_size, max=block_size)
    if ids.numel() != int(sizes.sum()):
        raise ValueError("selected IDs are not made of complete blocks")
    return blocks


def tile_block_lists(tile_blocks: Sequence[torch.Tensor], device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-tile block id lists -> (flat int32 ids, int32 offsets[n_tiles + 1]) on ``device``."""
    lists = [torch.as_tensor(b).flatten().to(torch.int32) for b in tile_blocks]
    counts = torch.tensor([0] + [b.numel() for b in lists], dtype=torch.int64)
    offsets = counts.cumsum(0).to(torch.int32)
    flat = torch.cat(lists) if lists else torch.empty(0, dtype=torch.int32)
    if flat.numel() == 0:
        flat = torch.zeros(1, dtype=torch.int32)
    return flat.to(device, non_blocking=True), offsets.to(device, non_blocking=True)


class PrefillWorkspace:
    """Zero-initialised scratch of qcc_indexed_ffn_prefill for one stream."""

    def __init__(self, device: torch.device, nbytes: int, stream: torch.cuda.Stream):
        lib = _lib.library()
        self.nbytes = nbytes
        self.buffer = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.status_offset = int(lib.qcc_prefill_workspace_status_offset())
        _lib.check(lib.qcc_workspace_init(self.buffer.data_ptr(), nbytes, stream.cuda_stream), "qcc_workspace_init")

    def read_status(self, clear: bool = True) -> int:
        word = self.buffer[self.status_offset:self.status_offset + 4]
        value = int(word.view(torch.int32).item())
        if clear and value:
            word.zero_()
        return value


class BlockSparsePrefill:
    """Prefill of one packed FFN layer (bf16, fp16 or fp32 records) over per-tile block selections."""

    def __init__(self, weights: PackedFFNWeights):
        if weights.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise ValueError(f"expected bf16, fp16 or fp32 records for the tensor-core prefill, got {weights.dtype}")
        _lib.require_cuda(weights.packed)
        self.weights = weights
        self._code = _lib.dtype_code(weights.dtype)
        self._workspaces: dict[int, PrefillWorkspace] = {}

    @property
    def hidden(self) -> int:
        return self.weights.hidden

    @property
    def n_blocks(self) -> int:
        return (self.weights.n_records + BLOCK_RECORDS - 1) // BLOCK_RECORDS

    def workspace(self, stream: torch.cuda.Stream) -> PrefillWorkspace:
        ws = self._workspaces.get(stream.cuda_stream)
        if ws is None:
            with torch.cuda.device(self.weights.device):
                nbytes = int(_lib.library().qcc_prefill_workspace_bytes(self.weights.n_records, self.hidden))
            if nbytes <= 0:
                raise ValueError("qcc_prefill_workspace_bytes rejected the layer shape")
            ws = PrefillWorkspace(self.weights.device, nbytes, stream)
            self._workspaces[stream.cuda_stream] = ws
        return ws

    def check(self) -> None:
        """Raise if a call flagged a device-side error since the last check (synchronises)."""
        for ws in self._workspaces.values():
            bits = ws.read_status()
            if bits & _lib.DEV_ID_RANGE:
                raise ValueError("selected block ID out of range")
            if bits & _lib.DEV_TIMEOUT:
                raise RuntimeError("qcc_indexed_ffn_prefill: a bounded wait ran out")

    def __call__(self, x: torch.Tensor, tile_blocks, **kwargs) -> torch.Tensor:
        return self.forward(x, tile_blocks, **kwargs)

    def forward(self, x: torch.Tensor, tile_blocks, *, out: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """y [T, H] for x [T, H].

        tile_blocks: a sequence of ceil(T / 128) 1-D block-id tensors (tile t
        covers tokens [128t, 128t + 128)), or a pair (flat int32 block ids,
        int32 offsets[n_tiles + 1]) already on the device.
        """
        w = self.weights
        if x.dim() != 2 or x.shape[1] != w.hidden:
            raise ValueError(f"expected x of shape [T, {w.hidden}], got {tuple(x.shape)}")
        if x.dtype != w.dtype:
            raise ValueError(f"expected x in {w.dtype}, got {x.dtype}")
        if x.stride(1) != 1 or (x.stride(0) * x.element_size()) % 16 != 0:
            raise ValueError("x must be contiguous along hidden with a 16-byte aligned row stride")
        _lib.require_cuda(x)
        n_tokens = x.shape[0]
        n_tiles = (n_tokens + TILE_TOKENS - 1) // TILE_TOKENS
        if isinstance(tile_blocks, tuple) and len(tile_blocks) == 2 and isinstance(tile_blocks[0], torch.Tensor) \
                and tile_blocks[0].is_cuda:
            flat, offsets = tile_blocks
            if flat.dtype != torch.int32 or offsets.dtype != torch.int32 or offsets.numel() != n_tiles + 1:
                raise ValueError(f"expected int32 block ids and {n_tiles + 1} int32 offsets")
        else:
            if len(tile_blocks) != n_tiles:
                raise ValueError(f"expected {n_tiles} per-tile block lists, got {len(tile_blocks)}")
            flat, offsets = tile_block_lists(tile_blocks, x.device)
        out_dtype = out_dtype or x.dtype
        if out is None:
            out = torch.empty((n_tokens, w.hidden), dtype=out_dtype, device=x.device)
        elif out.shape != (n_tokens, w.hidden) or out.stride(1) != 1:
            raise ValueError("out must be [T, hidden] and contiguous along hidden")
        stream = torch.cuda.current_stream(x.device)
        ws = self.workspace(stream)
        lib = _lib.library()
        _lib.check(lib.qcc_indexed_ffn_prefill(x.data_ptr(), x.stride(0), n_tokens, w.hidden, w.packed.data_ptr(),
                                               w.n_records, self._code, flat.data_ptr(), offsets.data_ptr(),
                                               ws.buffer.data_ptr(), ws.nbytes, out.data_ptr(), out.stride(0),
                                               _lib.dtype_code(out.dtype), stream.cuda_stream),
                   "qcc_indexed_ffn_prefill")
        return out
