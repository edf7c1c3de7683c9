"""Host-offload stager: an FFN layer whose cold neuron records live in pinned host RAM.

The reference stages whole layers synchronously from pageable memory
(integration/freetoken_qcc/low_vram/staging.py:43-67) and keeps a row gather
for a future neuron-level mode (host_store.py:24-26); its LRU cache exists
only as a host-side simulation (runtime/temporal.py:57-75).  Here one layer
keeps:

* an HBM resident array: the always-resident ("hot") records in slots
  [0, n_hot) and ``capacity`` cache slots after them;
* the remaining ("cold") records in a pinned host store;
* a device slot table and LRU list updated by ``qcc_cache_resolve``.

Per decode step (all device-side, no host round trip): resolve the step's
sorted ids into resident slots and misses; on a side stream copy the missed
records from the host store into their cache slots (``qcc_gather_records``,
reading host memory in place over PCIe) while the fused kernel runs over the
resident records; then a second fused call over the new slots adds onto that
partial result.
"""
from __future__ import annotations

import torch

from .. import _lib
from .engine import IndexedSparseFFN
from .packing import PackedFFNWeights

COUNT_NAMES = ("resident", "misses", "cache_hits", "evicted", "hot_hits", "overflow")


class HostOffloadLayer:
    """One packed FFN layer split between an HBM hot set + cache and a pinned host store."""

    def __init__(self, packed: torch.Tensor, hidden: int, hot_ids: torch.Tensor, capacity: int, max_k: int,
                 device: torch.device | str = "cuda"):
        """packed: [N, 3*Hp] records (CPU or CUDA); hot_ids: ids kept in HBM; capacity: cache slots."""
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("HostOffloadLayer needs a CUDA device (no CPU fallback)")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        n = packed.shape[0]
        hot_ids = torch.as_tensor(hot_ids, dtype=torch.long).cpu().sort().values
        is_hot = torch.zeros(n, dtype=torch.bool)
        is_hot[hot_ids] = True
        cold_ids = torch.nonzero(~is_hot).flatten()
        self.n_records, self.hidden, self.capacity, self.max_k = n, hidden, capacity, max_k
        self.n_hot = hot_ids.numel()
        self.device = device
        src = packed if packed.device.type == "cpu" else packed.to("cpu")
        self.resident = torch.zeros((self.n_hot + capacity, packed.shape[1]), dtype=packed.dtype, device=device)
        self.resident[:self.n_hot].copy_(src[hot_ids])
        self.cold_host = src[cold_ids].contiguous().pin_memory()
        slot_of = torch.full((n,), -1, dtype=torch.int32)
        slot_of[hot_ids] = torch.arange(self.n_hot, dtype=torch.int32)
        cold_index = torch.full((n,), -1, dtype=torch.int32)
        cold_index[cold_ids] = torch.arange(cold_ids.numel(), dtype=torch.int32)
        self.hot_ids = hot_ids
        self.slot_of = slot_of.to(device)
        self.cold_index = cold_index.to(device)
        self.owner = torch.full((capacity,), -1, dtype=torch.int32, device=device)
        self.last_use = torch.full((capacity,), -1, dtype=torch.int32, device=device)
        self.lru_order = torch.arange(capacity, dtype=torch.int32, device=device)  # least recently used first
        self.resident_ids = torch.empty(max(1, max_k), dtype=torch.int32, device=device)
        self.miss_slot = torch.empty(max(1, max_k), dtype=torch.int32, device=device)
        self.miss_src = torch.empty(max(1, max_k), dtype=torch.int32, device=device)
        self.counts = torch.zeros(len(COUNT_NAMES), dtype=torch.int32, device=device)
        self.engine = IndexedSparseFFN(PackedFFNWeights(self.resident, hidden, self.n_hot + capacity))
        self.copy_stream = torch.cuda.Stream(device)
        self.record_bytes = self.resident.shape[1] * self.resident.element_size()
        self.step = 0

    @classmethod
    def from_artefact(cls, root, hot_ids: torch.Tensor, capacity: int, max_k: int,
                      device: torch.device | str = "cuda", checksums: bool = True) -> "HostOffloadLayer":
        """A layer whose records come from a packed-record artefact (``runtime.artefact``).

        The reference's low-VRAM store loads its layers from a checksummed
        stream cache (integration/freetoken_qcc/low_vram/host_store.py:29-57);
        here the artefact's records are read once from disk into host memory,
        the hot set goes to HBM and the rest into the pinned host store.
        """
        from . import artefact

        manifest = artefact.load_manifest(root)
        artefact.validate_files(root, manifest, checksums)
        records = artefact.read_records(root, manifest)
        return cls(records, manifest["hidden"], hot_ids, capacity, max_k, device)

    @property
    def cold_bytes(self) -> int:
        return self.cold_host.numel() * self.cold_host.element_size()

    def stats(self) -> dict:
        """Counters of the last step (synchronises)."""
        return dict(zip(COUNT_NAMES, (int(v) for v in self.counts.tolist())))

    def __call__(self, x: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        return self.forward(x, ids)

    def forward(self, x: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        """y [B, H] for x [B, H] and sorted, unique int32 ids (every token uses every id)."""
        if ids.dtype != torch.int32 or ids.dim() != 1 or not ids.is_contiguous():
            raise ValueError("selected IDs must be contiguous one-dimensional int32")
        if ids.numel() > self.max_k:
            raise ValueError(f"expected at most {self.max_k} selected IDs, got {ids.numel()}")
        _lib.require_cuda(x, ids)
        lib = _lib.library()
        stream = torch.cuda.current_stream(self.device)
        k = ids.numel()
        _lib.check(lib.qcc_cache_resolve(ids.data_ptr(), k, None, self.slot_of.data_ptr(), self.n_records,
                                         self.n_hot, self.owner.data_ptr(), self.last_use.data_ptr(),
                                         self.lru_order.data_ptr(), self.capacity,
                                         self.cold_index.data_ptr(), self.step, self.resident_ids.data_ptr(),
                                         self.miss_slot.data_ptr(), self.miss_src.data_ptr(),
                                         self.counts.data_ptr(), stream.cuda_stream), "qcc_cache_resolve")
        self.step += 1
        resolved = torch.cuda.Event()
        resolved.record(stream)
        self.copy_stream.wait_event(resolved)
        _lib.check(lib.qcc_gather_records(self.cold_host.data_ptr(), self.record_bytes, self.miss_src.data_ptr(),
                                          self.miss_slot.data_ptr(), self.counts[1:2].data_ptr(), k,
                                          self.resident.data_ptr(), self.copy_stream.cuda_stream),
                   "qcc_gather_records")
        copied = torch.cuda.Event()
        copied.record(self.copy_stream)
        # Resident records run while the missed ones are still crossing PCIe.
        partial = self.engine(x, self.resident_ids[:max(1, k)], n_ids_dev=self.counts[0:1],
                              out_dtype=torch.float32)
        stream.wait_event(copied)
        return self.engine(x, self.miss_slot[:max(1, k)], n_ids_dev=self.counts[1:2], accumulate=partial,
                           out_dtype=x.dtype)
