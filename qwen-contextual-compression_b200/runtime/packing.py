"""Neuron-major packed FFN weights.

Record n of the packed array is ``[gate[n, :Hp] | up[n, :Hp] | down[:Hp, n]]``
(Hp = hidden rounded up to 8, zero padded), so one contiguous 3*Hp*esize-byte
read fetches everything neuron n contributes (30720 B for hidden 5120 bf16,
the per-neuron payload of reference runtime/temporal.py:55).  The reference
keeps three separate tensors and at most a transposed down copy
(runtime/weights.py:89-96).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _lib


def validate_weight_shapes(gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                           transposed_down: bool = False) -> tuple[int, int]:
    """Return (hidden, intermediate); same contract as runtime/weights.py:33-39.

    gate and up are [N, H]; down is [H, N] (or [N, H] when transposed_down).
    """
    if gate.ndim != 2 or up.ndim != 2 or down.ndim != 2:
        raise ValueError("FFN weights must all be matrices")
    n, h = gate.shape
    expected_down = (n, h) if transposed_down else (h, n)
    if tuple(up.shape) != (n, h) or tuple(down.shape) != expected_down:
        raise ValueError(f"Incompatible FFN shapes: gate={tuple(gate.shape)}, up={tuple(up.shape)}, "
                         f"down={tuple(down.shape)}")
    return h, n


@dataclass
class PackedFFNWeights:
    """A packed FFN layer (or one rank's contiguous slice of it) on one GPU."""

    packed: torch.Tensor      # [n_records, 3 * hidden_pad] in dtype
    hidden: int
    n_records: int
    record_offset: int = 0    # global id of record 0 (intermediate-dimension shards)
    intermediate: int | None = None  # full N of the unsharded layer

    def __post_init__(self):
        if self.intermediate is None:
            self.intermediate = self.n_records

    @property
    def dtype(self) -> torch.dtype:
        return self.packed.dtype

    @property
    def device(self) -> torch.device:
        return self.packed.device

    @property
    def hidden_pad(self) -> int:
        return (self.hidden + 7) // 8 * 8

    @property
    def record_bytes(self) -> int:
        return 3 * self.hidden_pad * self.packed.element_size()

    def record_slice(self, begin: int, end: int) -> "PackedFFNWeights":
        """Records [begin, end) as a view (ids local to the slice)."""
        return PackedFFNWeights(self.packed[begin:end], self.hidden, end - begin, self.record_offset + begin,
                                self.intermediate)


def pack_neuron_major(gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                      transposed_down: bool = False, record_range: tuple[int, int] | None = None) -> PackedFFNWeights:
    """Pack gate [N,H], up [N,H], down [H,N] (or down_t [N,H]) on their CUDA device.

    ``record_range=(begin, end)`` packs only neurons [begin, end), the slice an
    intermediate-dimension shard owns.
    """
    hidden, n = validate_weight_shapes(gate, up, down, transposed_down)
    device = _lib.require_cuda(gate, up, down)
    if gate.dtype != up.dtype or gate.dtype != down.dtype:
        raise TypeError("gate, up and down must share a dtype")
    code = _lib.dtype_code(gate.dtype)
    begin, end = record_range if record_range is not None else (0, n)
    if not 0 <= begin <= end <= n:
        raise ValueError(f"record range {record_range} outside [0, {n}]")
    gate = gate.contiguous()
    up = up.contiguous()
    down = down.contiguous()
    hp = (hidden + 7) // 8 * 8
    packed = torch.empty((end - begin, 3 * hp), dtype=gate.dtype, device=device)
    esize = gate.element_size()
    if transposed_down:   # down_t [N, H]: element (h, n) at n * H + h
        sh, sn = 1, hidden
        down_ptr = down.data_ptr() + begin * hidden * esize
    else:                 # down [H, N]: element (h, n) at h * N + n
        sh, sn = n, 1
        down_ptr = down.data_ptr() + begin * esize
    lib = _lib.library()
    with torch.cuda.device(device):
        status = lib.qcc_pack_records(gate.data_ptr() + begin * hidden * esize, up.data_ptr() + begin * hidden * esize,
                                      hidden, down_ptr, sh, sn, end - begin, hidden, code, packed.data_ptr(),
                                      _lib.stream_handle(device))
    _lib.check(status, "qcc_pack_records")
    return PackedFFNWeights(packed, hidden, end - begin, begin, n)
