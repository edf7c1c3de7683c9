"""Intermediate-dimension sharding across real GPUs, when at least two are visible.

Each rank packs only its record range and keeps its part of the global ids.
The cross-rank sum is either fused into the decode kernel (exchange buffers
over NVLink, CUDA IPC) or an NCCL all-reduce of fp32 partials; both must match
the oracle, the fused sum must be identical on every rank (rank-ordered) and
stable across repeated calls (rotating exchange slots).  Runs as spawned
child processes with a short process-group timeout, NVLS off; skipped on
machines with one GPU.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, queue) -> None:
    import datetime
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch.distributed as dist
    from oracle import ffn as offn
    import qcc_b200.workloads as workloads
    from qcc_b200.runtime.packing import PackedFFNWeights
    from qcc_b200.runtime.sharded import ShardedIndexedFFN, shard_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        hidden, n = 2048, 8192
        begin, end = shard_range(n, world, rank)
        layer = workloads.decode_layer(hidden=hidden, intermediate=n, device=device, seed=5, record_range=(begin, end))
        weights = PackedFFNWeights(layer.packed, hidden, end - begin, begin, n)
        fused = ShardedIndexedFFN(weights, group=dist.group.WORLD, allreduce="fused")
        nccl = ShardedIndexedFFN(weights, group=dist.group.WORLD, allreduce="nccl")
        k = workloads.retention_k(n, 0.25)
        ids = workloads.decode_ids(n, k, token=4).to(device)
        x = workloads.decode_x(hidden=hidden).to(device)
        y = fused(x, ids)
        y_nccl = nccl(x, ids)
        ys = [fused(x, ids) for _ in range(50)]  # rotating exchange slots, graph-free loop
        # The caller's output buffer (out=), fused and NCCL paths.
        y_out, y_nccl_out = torch.empty_like(y), torch.empty_like(y_nccl)
        fused(x, ids, out=y_out)
        nccl(x, ids, out=y_nccl_out)
        torch.cuda.synchronize(device)
        stable = all(torch.equal(y, yi) for yi in ys) and torch.equal(y_out, y) and torch.equal(y_nccl_out, y_nccl)
        other = torch.empty_like(y)
        dist.broadcast(other if rank else y.clone(), src=0)
        if rank:
            other_equal = torch.equal(other, y)
        else:
            other_equal = True
        # Calls alternating batch 4 and batch 1 on one exchange buffer (sized for
        # batch 4): slots are spaced by the buffer's size, so the batches never
        # overlap and every call returns what the first call of its batch did.
        x4 = workloads.decode_x(batch=4, hidden=hidden).to(device)
        first4, first1 = fused(x4, ids), fused(x4[:1], ids)
        alternating = True
        for i in range(8):
            if i % 2 == 0:
                alternating = alternating and torch.equal(fused(x4, ids), first4)
            else:
                alternating = alternating and torch.equal(fused(x4[:1], ids), first1)
        torch.cuda.synchronize(device)
        close = offn.rel_l2(first1.double().cpu().numpy(), first4[:1].double().cpu().numpy()) <= 1e-2
        flags = torch.tensor([int(stable), int(other_equal), int(alternating), int(close)], device=device)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        fused.engine.check()
        # Gather the full layer on rank 0 for the oracle (small layer).
        parts = [torch.empty_like(layer.packed) if r != rank else layer.packed for r in range(world)]
        sizes = [shard_range(n, world, r) for r in range(world)]
        gathered = None
        if rank == 0:
            gathered = [torch.empty((e - b, layer.packed.shape[1]), dtype=layer.packed.dtype, device=device)
                        for b, e in sizes]
        dist.gather(layer.packed, gathered if rank == 0 else None, dst=0)
        if rank == 0:
            full = torch.cat(gathered).cpu()
            gate, up, down = full[:, :hidden], full[:, hidden:2 * hidden], full[:, 2 * hidden:].t()
            expected = offn.sparse_ffn_f64(x.cpu(), ids.cpu(), gate, up, down)
            queue.put((offn.rel_l2(y.double().cpu().numpy(), expected),
                       offn.rel_l2(y_nccl.double().cpu().numpy(), expected), flags.tolist()))
        del parts
        fused.close()
        nccl.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_sharded_layer_matches_oracle():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    err_fused, err_nccl, flags = queue.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert err_fused <= 1e-2 and err_nccl <= 1e-2
    assert flags[:2] == [1, 1], "fused sum differs between ranks or between repeated calls"
    assert flags[2:] == [1, 1], "calls alternating batch 4 and batch 1 on one exchange buffer disagree"
