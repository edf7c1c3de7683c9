"""The decode's cross-rank exchange and its early-start flag, on one GPU.

* A bounded exchange wait runs out: a two-rank call whose "peer" buffer is a
  second local buffer that no rank ever fills.  The wait bound is set to a
  few milliseconds (``qcc_exchange_set_wait_limit``); the call must come back
  with QCC_DEV_TIMEOUT in the workspace status, without a fault or a hang,
  ``ShardedIndexedFFN.check`` must raise, and after ``qcc_exchange_init`` the
  same buffers serve a one-rank call again.  Nothing here waits for another
  launch: the only wait is on words that nothing writes, and it is bounded.
* ``ids_ready`` (QCC_IDS_READY) lets a decode launch start its record copies
  before the launches ahead of it finish; y must be bit-identical to the
  default path, back to back across layers and inside a CUDA graph.
* A batch change between calls on one exchange buffer keeps its slots apart
  (the slots are spaced by the buffer's size): two-rank calls at batch 4,
  1, 4, ... with the peer's sums filled in by the host.
"""
from __future__ import annotations

import ctypes
import time
from types import SimpleNamespace

import pytest
import torch

from oracle import ffn as offn
import qcc_b200.workloads as workloads
from qcc_b200 import _lib
from qcc_b200.runtime import IndexedSparseFFN
from qcc_b200.runtime.packing import PackedFFNWeights
from qcc_b200.runtime.sharded import ShardedIndexedFFN

pytestmark = pytest.mark.gpu


class _LocalBuffers:
    """Exchange buffers allocated in this process only (no IPC, no peer)."""

    def __init__(self, count: int, world: int, batch: int, hidden: int, dtype: torch.dtype):
        lib = _lib.library()
        self.nbytes = int(lib.qcc_exchange_bytes(world, batch, hidden, _lib.dtype_code(dtype)))
        self.ptrs = []
        for _ in range(count):
            p = ctypes.c_void_p()
            _lib.check(lib.qcc_exchange_alloc(self.nbytes, ctypes.byref(p)), "qcc_exchange_alloc")
            self.ptrs.append(p.value)

    def view(self, world: int, rank: int, order):
        ptrs = [self.ptrs[i] for i in order]
        return SimpleNamespace(world=world, rank=rank, nbytes=self.nbytes, pointers=(ctypes.c_void_p * world)(*ptrs))

    def close(self):
        lib = _lib.library()
        for p in self.ptrs:
            lib.qcc_exchange_free(p)
        self.ptrs = []


def test_exchange_wait_runs_out_and_reports_timeout():
    hidden, n = 1024, 2048
    device = torch.device("cuda", 0)
    layer = workloads.decode_layer(hidden=hidden, intermediate=n, device=device, seed=21)
    k = workloads.retention_k(n, 0.25)
    ids = workloads.decode_ids(n, k, token=1).to(device)
    x = workloads.decode_x(hidden=hidden).to(device)
    expected = IndexedSparseFFN(PackedFFNWeights(layer.packed, hidden, n))(x, ids)
    lib = _lib.library()
    bufs = _LocalBuffers(2, world=2, batch=1, hidden=hidden, dtype=torch.bfloat16)
    try:
        limit_ns = 20_000_000  # 20 ms
        _lib.check(lib.qcc_exchange_set_wait_limit(bufs.ptrs[0], limit_ns), "qcc_exchange_set_wait_limit")
        # Rank 0 of two: rank 1's sums never arrive in buffer 0.
        shard = ShardedIndexedFFN(PackedFFNWeights(layer.packed, hidden, n, 0, n), exchange=bufs.view(2, 0, [0, 1]))
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        shard(x, ids)
        torch.cuda.synchronize(device)
        elapsed = time.perf_counter() - t0
        assert elapsed < 1.5, f"the exchange wait took {elapsed:.3f} s against a 20 ms bound"
        with pytest.raises(RuntimeError, match="bounded wait ran out"):
            shard.check()
        # Recovery: re-initialise the buffer, then a one-rank call works again.
        _lib.check(lib.qcc_exchange_init(bufs.ptrs[0], bufs.nbytes), "qcc_exchange_init")
        single = ShardedIndexedFFN(PackedFFNWeights(layer.packed, hidden, n, 0, n), exchange=bufs.view(1, 0, [0]))
        y = single(x, ids)
        torch.cuda.synchronize(device)
        single.check()
        assert torch.equal(y, expected)
    finally:
        torch.cuda.synchronize(device)
        bufs.close()


class _DeviceBytes:
    """A raw device allocation seen as a torch uint8 tensor (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def test_exchange_slots_survive_batch_changes():
    """One buffer sized for batch 4 serves calls at batch 4, 1, 4, 1, ... (slots spaced by capacity).

    Two ranks, emulated on one GPU without a second launch: before each call
    the host fills rank 1's region of this rank's buffer with +0.0 sums (what
    a peer with no records would store), at the slot and offsets the buffer's
    size gives.  The call adds them to its own sums, re-marks the words empty
    and must return the plain decode bit for bit at every batch.
    """
    hidden, n, world = 2048, 4096, 2
    device = torch.device("cuda", 0)
    layer = workloads.decode_layer(hidden=hidden, intermediate=n, device=device, seed=22)
    engine = IndexedSparseFFN(PackedFFNWeights(layer.packed, hidden, n))
    k = workloads.retention_k(n, 0.25)
    ids = workloads.decode_ids(n, k, token=2).to(device)
    x4 = workloads.decode_x(batch=4, hidden=hidden).to(device)
    bufs = _LocalBuffers(2, world=world, batch=4, hidden=hidden, dtype=torch.bfloat16)
    try:
        mine = torch.as_tensor(_DeviceBytes(bufs.ptrs[0], bufs.nbytes), device=device)
        words = mine[256:].view(torch.int32)
        slot_words = (bufs.nbytes - 256) // (3 * world * 16)
        shard = ShardedIndexedFFN(PackedFFNWeights(layer.packed, hidden, n, 0, n),
                                  exchange=bufs.view(world, 0, [0, 1]))
        want = {4: engine(x4, ids), 1: engine(x4[:1], ids)}
        for call in range(12):
            batch = 4 if call % 2 == 0 else 1
            nvec = batch * hidden // 4
            slot = call % 3
            first = ((slot * world + 1) * slot_words) * 4  # int32 index of rank 1's region
            words[first:first + 4 * nvec].zero_()
            y = shard(x4[:batch], ids)
            assert torch.equal(y, want[batch]), f"call {call} (batch {batch})"
        torch.cuda.synchronize(device)
        shard.check()
        # Every column-sum word is the empty mark again.
        assert bool((words == -2**31).all())
        assert int(mine[:4].view(torch.int32).item()) == 12  # the buffer counted its launches
    finally:
        torch.cuda.synchronize(device)
        bufs.close()


@pytest.mark.parametrize("retention", [0.25, 0.02])
def test_ids_ready_is_bit_identical_back_to_back(retention):
    hidden, n, layers = 5120, 8192, 3
    device = torch.device("cuda", 0)
    engines = [IndexedSparseFFN(PackedFFNWeights(workloads.decode_layer(hidden=hidden, intermediate=n,
                                                                         device=device, seed=30 + s).packed,
                                                 hidden, n)) for s in range(layers)]
    k = workloads.retention_k(n, retention)
    steps = 9
    ids = torch.stack([workloads.decode_ids(n, k, token=t) for t in range(steps)]).to(device)
    x = workloads.decode_x(hidden=hidden).to(device)
    plain = torch.empty((steps, 1, hidden), dtype=torch.bfloat16, device=device)
    early = torch.empty_like(plain)
    for t in range(steps):
        engines[t % layers](x, ids[t], out=plain[t])
    for t in range(steps):
        engines[t % layers](x, ids[t], out=early[t], ids_ready=True)
    torch.cuda.synchronize(device)
    assert torch.equal(plain, early)
    # The same sequence captured in one CUDA graph.
    graphed = torch.empty_like(plain)
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for t in range(steps):
            engines[t % layers](x, ids[t], out=graphed[t], ids_ready=True)
    graph.replay()
    torch.cuda.synchronize(device)
    assert torch.equal(plain, graphed)
    # And against the oracle, for one step.
    layer0 = workloads.decode_layer(hidden=hidden, intermediate=n, device=device, seed=30)
    want = offn.sparse_ffn_f64(x.cpu(), ids[0].cpu(), layer0.gate().cpu(), layer0.up().cpu(), layer0.down().cpu())
    assert offn.rel_l2(early[0].double().cpu().numpy(), want) <= 1e-2
    for e in engines:
        e.check()
