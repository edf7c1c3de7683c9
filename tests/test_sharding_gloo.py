"""Host-side sharding logic across real processes (gloo on CPU, world size 2 and 4).

Each rank takes its contiguous record range, keeps the global ids inside it
(rebased) and computes its partial y with the oracle; an all-reduce of the
partials must equal the unsharded layer.  The CUDA kernels are replaced by
the oracle here; the GPU tests cover them.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, queue) -> None:
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from oracle import ffn as offn
    from oracle import select as osel
    from qcc_b200.runtime.sharded import shard_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(5)
        h, n, batch = 64, 200, 3
        gate, up, down = torch.randn(n, h, generator=gen), torch.randn(n, h, generator=gen), torch.randn(h, n, generator=gen)
        x = torch.randn(batch, h, generator=gen)
        scores = torch.randn(batch, n, generator=gen)
        rows = osel.topk_ids(scores.numpy(), 50)  # identical on every rank (deterministic selector)
        b, e = shard_range(n, world, rank)
        local, mask = osel.union_with_mask(rows, b, e)
        local_t = torch.from_numpy(local.astype("int64"))
        part = torch.from_numpy(offn.sparse_ffn_f64(x, local_t, gate[b:e], up[b:e], down[:, b:e],
                                                    token_mask=torch.from_numpy(mask)))
        dist.all_reduce(part)
        full = torch.stack([torch.from_numpy(offn.sparse_ffn_f64(x[t:t + 1], torch.from_numpy(rows[t]).long(),
                                                                 gate, up, down))[0] for t in range(batch)])
        queue.put((rank, float((part - full).abs().max()), (b, e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_sharded_partials_sum_to_full(world):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ranges = sorted(r[2] for r in results)
    assert ranges[0][0] == 0 and ranges[-1][1] == 200
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
    assert max(r[1] for r in results) < 1e-9


def test_shard_range_partition():
    from qcc_b200.runtime.sharded import shard_range
    for n in (17408, 17, 5):
        for world in (1, 2, 4, 8):
            pieces = [shard_range(n, world, r) for r in range(world)]
            assert pieces[0][0] == 0 and pieces[-1][1] == n
            assert all(pieces[i][1] == pieces[i + 1][0] for i in range(world - 1))
    assert shard_range(17408, 8, 3) == (6528, 8704)
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)
