"""Intermediate-dimension sharding of one FFN layer over GPUs (one process per GPU).

Rank r of P owns the contiguous records [r*N//P, (r+1)*N//P).  Every rank
holds the same global selected ids (the selector is deterministic and
replicated, its output ascending) and keeps the ones inside its range,
rebased: for one id list shared by all tokens the decode kernel finds that
run itself; per-token id rows first go through qcc_build_union (one small
launch: union plus token mask).  The sum over ranks is
either fused into that kernel (``allreduce="fused"``, the default: each CTA
stores its column sums into every rank's exchange buffer over NVLink and adds
the ranks' sums in rank order -- no NCCL call, no extra launch) or an NCCL
all-reduce of the fp32 partials followed by a cast (``allreduce="nccl"``).
Only y (hidden fp32 values per token, 20 KB at hidden 5120) crosses NVLink.
The reference has no distributed path
(integration/freetoken_qcc/low_vram/adapter.py:106-107 refuses TP != 1).
"""
from __future__ import annotations

import torch

from .. import _lib
from .engine import IndexedSparseFFN
from .packing import PackedFFNWeights
from .selector import build_union


def shard_range(intermediate: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous record range of `rank` among `world` shards."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return intermediate * rank // world, intermediate * (rank + 1) // world


class PeerExchange:
    """The exchange buffers of all ranks of a process group, mapped into this process.

    Each rank allocates one buffer (``qcc_exchange_bytes``), shares its CUDA
    IPC handle through the process group, and maps the other ranks' buffers.
    Collective: every rank of the group constructs it.  ``wait_limit_ns``
    bounds each wait for the other ranks' sums (None: the library's 2 s).
    """

    def __init__(self, group, device: torch.device, batch: int, hidden: int, dtype: torch.dtype,
                 wait_limit_ns: int | None = None):
        import ctypes
        import torch.distributed as dist

        lib = _lib.library()
        self.group = group
        self.wait_limit_ns = wait_limit_ns
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = int(lib.qcc_exchange_bytes(self.world, batch, hidden, _lib.dtype_code(dtype)))
        if self.nbytes == 0:
            raise ValueError("qcc_exchange_bytes rejected the world / batch / hidden")
        with torch.cuda.device(device):
            local = ctypes.c_void_p()
            _lib.check(lib.qcc_exchange_alloc(self.nbytes, ctypes.byref(local)), "qcc_exchange_alloc")
            self._local = local.value
            if wait_limit_ns is not None:
                _lib.check(lib.qcc_exchange_set_wait_limit(self._local, int(wait_limit_ns)),
                           "qcc_exchange_set_wait_limit")
            handle = (ctypes.c_uint8 * 64)()
            _lib.check(lib.qcc_ipc_handle(self._local, handle), "qcc_ipc_handle")
            mine = torch.tensor(list(handle), dtype=torch.uint8, device=device)
            gathered = torch.empty(self.world * 64, dtype=torch.uint8, device=device)
            dist.all_gather_into_tensor(gathered, mine, group=group)
            rows = gathered.view(self.world, 64).cpu()
            self._opened = []
            ptrs = []
            for q in range(self.world):
                if q == self.rank:
                    ptrs.append(self._local)
                    continue
                h = (ctypes.c_uint8 * 64)(*rows[q].tolist())
                p = ctypes.c_void_p()
                _lib.check(lib.qcc_ipc_open(h, ctypes.byref(p)), "qcc_ipc_open")
                self._opened.append(p.value)
                ptrs.append(p.value)
        self.pointers = (ctypes.c_void_p * self.world)(*ptrs)
        self.device = device

    def reset(self) -> None:
        """Re-initialise every rank's buffer after a timed-out exchange (collective).

        Every rank calls it between steps, with none of its exchange calls in
        flight; the barriers keep any rank from writing into a buffer that its
        owner has not re-initialised yet.
        """
        import torch.distributed as dist

        lib = _lib.library()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            _lib.check(lib.qcc_exchange_init(self._local, self.nbytes), "qcc_exchange_init")
            if self.wait_limit_ns is not None:
                _lib.check(lib.qcc_exchange_set_wait_limit(self._local, int(self.wait_limit_ns)),
                           "qcc_exchange_set_wait_limit")
        dist.barrier(group=self.group)

    def close(self) -> None:
        lib = _lib.library()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.qcc_ipc_close(p)
            self._opened = []
            if self._local:
                lib.qcc_exchange_free(self._local)
                self._local = None


class ShardedIndexedFFN:
    """One rank's slice of an indexed sparse FFN layer plus the cross-rank sum."""

    def __init__(self, weights: PackedFFNWeights, group=None, allreduce: str = "fused",
                 exchange: PeerExchange | None = None):
        if allreduce not in ("fused", "nccl"):
            raise ValueError("allreduce must be 'fused' or 'nccl'")
        self.weights = weights
        self.engine = IndexedSparseFFN(weights)
        self.group = group
        self.begin = weights.record_offset
        self.end = weights.record_offset + weights.n_records
        self.allreduce = allreduce if (group is not None or exchange is not None) else "nccl"
        self._own_exchange = False
        self.exchange = exchange
        if self.allreduce == "fused" and self.exchange is None:
            self.exchange = PeerExchange(group, weights.device, self.engine.max_batch, weights.hidden, weights.dtype)
            self._own_exchange = True

    def partial(self, x: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        """fp32 partial y of this rank's records; ids are global ([K] shared or [B, K] per token)."""
        rows = ids if ids.ndim == 2 else ids.unsqueeze(0)
        if rows.dtype != torch.int32:
            rows = rows.to(torch.int32)
        rows = rows.contiguous()
        local, mask, count = build_union(rows, self.begin, self.end)
        per_token = ids.ndim == 2
        x2 = x if x.ndim == 2 else x.unsqueeze(0)
        return self.engine(x2, local, token_mask=mask if per_token else None, n_ids_dev=count,
                           out_dtype=torch.float32)

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, ids_ready: bool = False,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        return self.forward(x, ids, ids_ready=ids_ready, out=out)

    def forward(self, x: torch.Tensor, ids: torch.Tensor, ids_ready: bool = False,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """y of the whole layer on every rank; ``ids_ready`` as in ``IndexedSparseFFN.forward``
        (used with one shared 1-D id list and the fused sum).  ``out``: optional [B, hidden] (or
        [hidden]) tensor in the weight dtype that receives y."""
        x2 = x if x.ndim == 2 else x.unsqueeze(0)
        out2 = None if out is None else (out if out.ndim == 2 else out.unsqueeze(0))
        if self.allreduce == "fused" and ids.ndim == 1:
            # One id list for every token: the kernel finds this shard's run.
            y = self.engine(x2, ids, exchange=self.exchange, id_range=(self.begin, self.end), ids_ready=ids_ready,
                            out=out2)
            return y if x.ndim == 2 else y.squeeze(0)
        if self.allreduce == "fused":
            rows = ids if ids.ndim == 2 else ids.unsqueeze(0)
            if rows.dtype != torch.int32:
                rows = rows.to(torch.int32)
            local, mask, count = build_union(rows.contiguous(), self.begin, self.end)
            y = self.engine(x2, local, token_mask=mask if ids.ndim == 2 else None, n_ids_dev=count,
                            exchange=self.exchange, out=out2)
            return y if x.ndim == 2 else y.squeeze(0)
        y32 = self.partial(x, ids)
        if self.group is not None:
            torch.distributed.all_reduce(y32, group=self.group)
        if out2 is None:
            out2 = torch.empty(y32.shape, dtype=self.weights.dtype, device=y32.device)
        elif out2.shape != y32.shape or out2.dtype != self.weights.dtype or not out2.is_contiguous():
            raise ValueError("out must be a contiguous [batch, hidden] tensor in the weight dtype")
        lib = _lib.library()
        _lib.check(lib.qcc_cast_f32(y32.data_ptr(), out2.data_ptr(), y32.numel(), _lib.dtype_code(out2.dtype),
                                    _lib.stream_handle(y32.device)), "qcc_cast_f32")
        return out2 if x.ndim == 2 else out2.squeeze(0)

    def check(self) -> None:
        """Raise if a call since the last check flagged a device-side error (host sync).

        ``RuntimeError`` when a bounded wait ran out -- with the fused sum, the
        other ranks' column sums did not arrive in time, y of that call is
        incomplete, and every rank must call :meth:`recover` before the next
        step; ``ValueError`` for a selected id outside the layer.
        """
        self.engine.check()

    def recover(self) -> None:
        """Clear the device status and re-initialise the exchange buffers (collective)."""
        for ws in list(self.engine._streams_ws.values()):
            ws.read_status(clear=True)
        if self.exchange is not None:
            self.exchange.reset()

    def close(self) -> None:
        if self._own_exchange and self.exchange is not None:
            self.exchange.close()
        self.exchange = None
        self.engine = None
